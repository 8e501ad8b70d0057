"""CPU tests of the oracle (oracle/gpt2_oracle.c): pinned against the golden
fixtures made by transformers' GPT2LMHeadModel (tests/golden/make_golden.py),
the published Philox4x32-10 known-answer vectors, and its own invariants."""
import numpy as np
import pytest

from helpers import attendable_rows, bert_golden_files, golden_files, load_bert_golden, load_golden, load_oracle

O = load_oracle()


# Philox4x32-10 known-answer vectors published with Random123 (kat_vectors:
# "philox4x32 10 <ctr x4> <key x2> <out x4>").
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_known_answers(ctr, key, want):
    assert tuple(int(x) for x in O.philox(ctr, key)) == want


def test_normal_fill_statistics_and_determinism():
    a = O.normal_fill(1 << 20, seed=5, stream=3)
    b = O.normal_fill(1 << 20, seed=5, stream=3)
    c = O.normal_fill(1 << 20, seed=5, stream=4)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    assert abs(a.mean()) < 5e-3 and abs(a.std() - 1.0) < 5e-3
    # a prefix of a longer fill is the shorter fill (element i depends on i only)
    assert np.array_equal(O.normal_fill(1001, 5, 3), a[:1001])


def test_token_ids_range():
    ids = O.token_ids(4, 1000, seed=1, vocab=50257)
    assert ids.min() >= 0 and ids.max() < 50257
    assert len(np.unique(ids)) > 3500


@pytest.mark.parametrize("path", golden_files(), ids=lambda p: p.split("/")[-1])
def test_oracle_matches_transformers(path):
    """FP32 logits of the oracle vs HF GPT2LMHeadModel on the same seeded weights: 1e-4 absolute
    (the reference's own tolerance, src/compare_outputs.py:17); observed about 3e-6."""
    shape, z = load_golden(path)
    blob = O.seeded_blob(shape, int(z["seed"]), int(z["init_mode"]))
    assert np.array_equal(blob[:16], z["blob_head"]), "seeded generator drifted"
    assert abs(blob.astype(np.float64).sum() - float(z["blob_sum"])) <= 1e-9 * max(1.0, abs(float(z["blob_sum"])))
    logits = O.forward(shape, blob, z["ids"], z["mask"])
    if "cols" in z:
        logits = logits[..., z["cols"]]
    err = np.abs(logits - z["logits"])
    assert err.max() <= 1e-4, err.max()
    # every row, including rows with no attendable key, matches
    rows = attendable_rows(z["mask"])
    assert err[~rows].max(initial=0.0) <= 1e-4


def test_oracle_thread_split_is_bitwise_identical():
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 3, 1)
    ids = O.token_ids(3, 40, 3, shape.vocab_size)
    mask = np.ones_like(ids)
    mask[1, :7] = 0
    O.set_loop_threads(1)
    a = O.forward(shape, blob, ids, mask)
    O.set_loop_threads(4)
    b = O.forward(shape, blob, ids, mask)
    O.set_loop_threads(1)
    assert np.array_equal(a, b)


def test_oracle_batch_invariance():
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 4, 1)
    ids = O.token_ids(3, 17, 4, shape.vocab_size)
    full = O.forward(shape, blob, ids)
    one = O.forward(shape, blob, ids[1:2])
    assert np.allclose(full[1:2], one, atol=1e-6)


def test_oracle_rejects_bad_inputs():
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 4, 0)
    with pytest.raises(ValueError):
        O.forward(shape, blob, np.array([[0, shape.vocab_size]]))
    with pytest.raises(ValueError):
        O.forward(shape, blob, np.array([[-1, 0]]))
    with pytest.raises(ValueError):
        O.forward(shape, blob, np.zeros((1, shape.n_positions + 1), dtype=np.int64))


@pytest.mark.parametrize("path", bert_golden_files(), ids=lambda p: p.split("/")[-1])
def test_bert_oracle_matches_transformers(path):
    """BERT encoder (src/bert-base-uncased/lower_bert_model.py:7-18): last_hidden_state and
    pooler_output of the oracle vs HF BertModel on the same seeded weights, within 1e-4."""
    shape, z = load_bert_golden(path)
    blob = O.bert_seeded_blob(shape, int(z["seed"]), int(z["init_mode"]))
    assert np.array_equal(blob[:16], z["blob_head"]), "seeded generator drifted"
    hidden, pooled = O.bert_forward(shape, blob, z["ids"], z["token_type_ids"], z["mask"])
    assert np.abs(hidden - z["hidden"]).max() <= 1e-4
    assert np.abs(pooled - z["pooled"]).max() <= 1e-4
