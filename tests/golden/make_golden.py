"""Generates the golden fixtures in tests/golden/ by running transformers'
GPT2LMHeadModel (the model that src/gpt/lower_gpt_model.py:20-50 and
src/gpt/pytorch_ref.py:16-33 of the reference export and check) on weights
produced by the seeded Philox generator of oracle/gpt2_oracle.c.

Run in a container that has transformers (no network or pretrained weights
needed):  python tests/golden/make_golden.py

Each fixture .npz holds the case's model shape, seed, init mode, ids, mask,
a weight checksum (to catch generator drift) and HF's FP32 logits (full, or
a fixed column subset plus the per-position top-5 of the full row when the
full logits would make the fixture large).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

SUBSET_COLS = np.concatenate([np.arange(0, 2048), np.arange(50257 - 64, 50257)])


def hf_model(shape: O.ModelShape, blob: np.ndarray):
    from transformers import GPT2Config, GPT2LMHeadModel
    cfg = GPT2Config(n_layer=shape.n_layer, n_embd=shape.n_embd, n_head=shape.n_head, n_inner=shape.n_inner,
                     vocab_size=shape.vocab_size, n_positions=shape.n_positions,
                     layer_norm_epsilon=shape.layer_norm_eps, activation_function="gelu_new",
                     resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0, tie_word_embeddings=True,
                     attn_implementation="eager")
    model = GPT2LMHeadModel(cfg).eval()
    off = O.blob_layout(shape)
    sd = model.state_dict()
    new = {}
    for i, name in enumerate(O.tensor_names(shape)):
        t = torch.from_numpy(blob[off[i]:off[i + 1]].copy()).reshape(sd[name].shape)
        new[name] = t
    new["lm_head.weight"] = new["transformer.wte.weight"]
    missing, unexpected = model.load_state_dict(new, strict=False)
    assert not unexpected, unexpected
    assert all(m.endswith(("attn.bias", "attn.masked_bias")) for m in missing), missing
    assert model.lm_head.weight.data_ptr() == model.transformer.wte.weight.data_ptr() or torch.equal(
        model.lm_head.weight, model.transformer.wte.weight)
    return model


def run_case(name, shape, seed, init_mode, ids, mask, subset=False):
    blob = O.seeded_blob(shape, seed, init_mode)
    model = hf_model(shape, blob)
    with torch.no_grad():
        logits = model(input_ids=torch.from_numpy(ids), attention_mask=torch.from_numpy(mask)).logits
    logits = logits.float().numpy()
    rec = dict(
        shape=np.array([shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                        shape.n_positions], dtype=np.int64),
        eps=np.float32(shape.layer_norm_eps), seed=np.uint64(seed), init_mode=np.int64(init_mode),
        ids=ids, mask=mask,
        blob_sum=np.float64(blob.astype(np.float64).sum()), blob_head=blob[:16].copy(),
        top5_idx=np.argsort(-logits, axis=-1, kind="stable")[..., :5].astype(np.int64),
    )
    rec["top5_val"] = np.take_along_axis(logits, rec["top5_idx"], axis=-1)
    if subset:
        rec["cols"] = SUBSET_COLS.astype(np.int64)
        rec["logits"] = np.ascontiguousarray(logits[..., SUBSET_COLS])
    else:
        rec["logits"] = logits
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **rec)
    print(f"wrote {path}: logits {rec['logits'].shape}")


def hf_bert(shape: O.BertShape, blob: np.ndarray):
    from transformers import BertConfig, BertModel
    cfg = BertConfig(vocab_size=shape.vocab_size, hidden_size=shape.n_embd, num_hidden_layers=shape.n_layer,
                     num_attention_heads=shape.n_head, intermediate_size=shape.n_inner,
                     max_position_embeddings=shape.n_positions, type_vocab_size=shape.type_vocab,
                     layer_norm_eps=shape.layer_norm_eps, hidden_act="gelu", hidden_dropout_prob=0.0,
                     attention_probs_dropout_prob=0.0, attn_implementation="eager")
    model = BertModel(cfg).eval()
    off = O.bert_blob_layout(shape)
    sd = model.state_dict()
    new = {n: torch.from_numpy(blob[off[i]:off[i + 1]].copy()).reshape(sd[n].shape)
           for i, n in enumerate(O.bert_tensor_names(shape))}
    missing, unexpected = model.load_state_dict(new, strict=False)
    assert not unexpected and not missing, (missing, unexpected)
    return model


def run_bert_case(name, shape, seed, init_mode, ids, tt, mask):
    blob = O.bert_seeded_blob(shape, seed, init_mode)
    model = hf_bert(shape, blob)
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(ids), token_type_ids=torch.from_numpy(tt),
                    attention_mask=torch.from_numpy(mask))
    rec = dict(
        shape=np.array([shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                        shape.n_positions, shape.type_vocab], dtype=np.int64),
        eps=np.float32(shape.layer_norm_eps), seed=np.uint64(seed), init_mode=np.int64(init_mode),
        ids=ids, token_type_ids=tt, mask=mask, blob_sum=np.float64(blob.astype(np.float64).sum()),
        blob_head=blob[:16].copy(), hidden=out.last_hidden_state.float().numpy(),
        pooled=out.pooler_output.float().numpy())
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **rec)
    print(f"wrote {path}: hidden {rec['hidden'].shape}")


def main_bert():
    tiny, base = O.BERT_TINY, O.BERT_BASE
    # The reference BERT host program's call (src/bert-base-uncased/call_bert.cpp:61-64), seeded weights.
    ids = np.array([[101, 2023, 2003, 1037, 7099, 7953, 2005, 14324, 2944, 9167, 1012, 102]], dtype=np.int64)
    run_bert_case("bert_base_refcall", base, 1234, 0, ids, np.zeros_like(ids), np.ones_like(ids))
    # BERT-base, right-padded batch (the benchmark's mask shape), token types 0 / 1 halves.
    ids = O.token_ids(2, 64, 33, base.vocab_size, stream=O.BERT_IDS_STREAM)
    tt = np.zeros_like(ids)
    tt[:, 32:] = 1
    mask = np.ones_like(ids)
    mask[1, 40:] = 0
    run_bert_case("bert_base_padded", base, 33, 1, ids, tt, mask)
    # Tiny model of the same family: every kind of mask, random token types.
    ids = O.token_ids(4, 23, 5, tiny.vocab_size, stream=O.BERT_IDS_STREAM)
    tt = O.token_ids(4, 23, 6, 2, stream=O.BERT_IDS_STREAM + 1)
    mask = np.ones_like(ids)
    mask[1, 12:] = 0
    mask[2, :] = 0
    mask[3, ::3] = 0
    run_bert_case("bert_tiny_masks", tiny, 5, 1, ids, tt, mask)


def main():
    torch.manual_seed(0)
    small, tiny = O.GPT2_SMALL, O.GPT2_TINY
    ones = lambda b, s: np.ones((b, s), dtype=np.int64)  # noqa: E731

    # The reference host program's own call: "The capital of France is"
    # (src/gpt/gpt2_call.cpp:54-55), B=1, S=5, all-ones mask; seeded weights.
    ref_ids = np.array([[464, 3139, 286, 4881, 318]], dtype=np.int64)
    run_case("gpt2_small_refcall", small, 1234, 0, ref_ids, ones(1, 5))

    # GPT-2 small, B=1, S=5, seeded ids (the CPU-runnable case).
    run_case("gpt2_small_cfg0", small, 1234, 0, O.token_ids(1, 5, 1234, small.vocab_size), ones(1, 5))

    # Every tensor random (biases, gains, shifts), B=2, S=9, a left-padded row.
    ids = O.token_ids(2, 9, 77, small.vocab_size)
    mask = ones(2, 9)
    mask[1, :3] = 0
    run_case("gpt2_small_random_padded", small, 77, 1, ids, mask, subset=True)

    # Tiny model of the same family: masks of every kind.
    B, S = 5, 23
    ids = O.token_ids(B, S, 9, tiny.vocab_size)
    mask = ones(B, S)
    mask[1, :5] = 0            # left padding: rows 0..4 attend to nothing
    mask[2, 7:11] = 0          # holes in the middle
    mask[2, -2:] = 0           # right padding
    mask[3, :] = 0             # nothing attendable anywhere
    mask[4, ::2] = 0           # every other key masked, row 0 fully masked
    run_case("tiny_random_masks", tiny, 9, 1, ids, mask)

    # Tiny model, S=1 and the full context S=P.
    run_case("tiny_random_s1", tiny, 10, 1, O.token_ids(3, 1, 10, tiny.vocab_size), ones(3, 1))
    run_case("tiny_random_fullctx", tiny, 11, 1, O.token_ids(2, tiny.n_positions, 11, tiny.vocab_size),
             ones(2, tiny.n_positions))


if __name__ == "__main__":
    which = sys.argv[1:] or ["gpt2", "bert"]
    if "gpt2" in which:
        main()
    if "bert" in which:
        main_bert()
