"""Incremental decoding with a KV cache (gpt2_kv_reserve / gpt2_prefill /
gpt2_decode_step / gpt2_generate) against the oracle's full forward.

The reference generates by re-running the whole forward on the grown
sequence and taking logits[:, -1] (src/gpt/lower_gpt_model.py:190-198,
src/gpt/run_gpt.py:20-24).  So the logits of decode step i must equal the
oracle's full-forward logits at position S + i - 1 of the same sequence:
FP32 within 1e-4 absolute; BF16 and FP8 weights (against the oracle on the
dequantized weights) by the stated bounds of helpers.top5_check, over the
prefill's and every step's positions together."""
import numpy as np
import pytest

from helpers import BF16_MAX_REL, BF16_TOP5_BOUND_REL, FP8_DEQ_MAX_REL, load_oracle, load_pkg, shape_to_cfg, top5_check

pytestmark = pytest.mark.gpu
pkg = load_pkg()
O = load_oracle()

FP32_ATOL = 1e-4
MAX_REL = {1: BF16_MAX_REL, 2: FP8_DEQ_MAX_REL}


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    t.cuda.set_device(0)
    return t


def _check(ref, got, dtype, label, seen):
    if dtype == 0:
        err = float(np.abs(got - ref).max())
        assert err <= FP32_ATOL, (label, err)
        return
    seen.append((ref, got))


@pytest.mark.parametrize("dtype,shape_name,B,S,steps", [(0, "GPT2_TINY", 3, 10, 6), (1, "GPT2_TINY", 4, 17, 5),
                                                         (2, "GPT2_TINY", 2, 9, 4), (0, "GPT2_SMALL", 1, 12, 3),
                                                         (1, "GPT2_SMALL", 16, 40, 3)])
def test_prefill_and_decode_steps_match_full_forward(torch, dtype, shape_name, B, S, steps):
    shape = getattr(O, shape_name)
    blob = O.seeded_blob(shape, 50 + S, 1)
    pkg.init(shape_to_cfg(pkg, shape, dtype), 0)
    pkg.load_weights(blob)
    ref_blob = O.fp8_dequantized_blob(shape, blob) if dtype == 2 else blob
    V = shape.vocab_size
    ld = (V + 3) // 4 * 4
    seq = O.token_ids(B, S + steps, 60 + S, V)
    st = torch.cuda.current_stream().cuda_stream
    pkg.kv_reserve(B, S + steps)
    ids = torch.from_numpy(np.ascontiguousarray(seq[:, :S])).cuda()
    logits = torch.empty(B, ld, device="cuda")
    pkg.prefill(ids.data_ptr(), B, S, logits.data_ptr(), ld, st)
    torch.cuda.synchronize()
    assert pkg.kv_length() == S
    full = O.forward(shape, ref_blob, seq)
    seen = []
    _check(full[:, S - 1], logits[:, :V].cpu().numpy(), dtype, f"prefill dtype {dtype}", seen)
    for i in range(steps):
        tok = torch.from_numpy(np.ascontiguousarray(seq[:, S + i])).cuda()
        pkg.decode_step(tok.data_ptr(), B, logits.data_ptr(), ld, st)
        torch.cuda.synchronize()
        _check(full[:, S + i], logits[:, :V].cpu().numpy(), dtype, f"step {i} dtype {dtype}", seen)
    if seen:
        top5_check(f"prefill + {steps} decode steps, dtype {dtype}, {shape_name} B{B}",
                   np.concatenate([r for r, _ in seen]), np.concatenate([g for _, g in seen]),
                   max_rel=MAX_REL[dtype], bound_rel=BF16_TOP5_BOUND_REL)
    assert pkg.kv_length() == S + steps
    assert pkg.status() == 0


def test_generate_is_the_oracle_greedy_chain(torch):
    """gpt2_generate (FP32) continues each prompt with the oracle's greedy argmax chain, compared
    step by step while the oracle's top-1 leads the runner-up by more than the FP32 tolerance."""
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 71, 1)
    pkg.init(shape_to_cfg(pkg, shape, 0), 0)
    pkg.load_weights(blob)
    B, S, n_new = 2, 6, 10
    prompt = O.token_ids(B, S, 71, shape.vocab_size)
    got = pkg.generate(prompt, n_new)
    assert got.shape == (B, n_new)
    for b in range(B):
        seq = prompt[b:b + 1].copy()
        for i in range(n_new):
            last = O.forward(shape, blob, seq)[0, -1]
            top2 = np.sort(last)[-2:]
            if top2[1] - top2[0] <= 4 * FP32_ATOL:
                break  # a near tie: either choice is the reference's within tolerance
            want = int(np.argmax(last))
            assert got[b, i] == want, (b, i)
            seq = np.concatenate([seq, [[want]]], axis=1)


def test_decode_errors_are_reported(torch):
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 72, 0)
    pkg.init(shape_to_cfg(pkg, shape, 1), 0)
    pkg.load_weights(blob)
    with pytest.raises(pkg.Gpt2Error):
        pkg.kv_reserve(17, 10)  # more than 16 sequences
    with pytest.raises(pkg.Gpt2Error):
        pkg.kv_reserve(2, shape.n_positions + 1)
    pkg.kv_reserve(2, 4)
    V = shape.vocab_size
    logits = torch.empty(2, V, device="cuda")
    tok = torch.zeros(2, dtype=torch.int64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(pkg.Gpt2Error, match="prefill first"):
        pkg.decode_step(tok.data_ptr(), 2, logits.data_ptr(), V, st)
    ids = torch.zeros(2, 3, dtype=torch.int64, device="cuda")
    pkg.prefill(ids.data_ptr(), 2, 3, logits.data_ptr(), V, st)
    pkg.decode_step(tok.data_ptr(), 2, logits.data_ptr(), V, st)
    with pytest.raises(pkg.Gpt2Error):  # the cache holds 4 positions
        pkg.decode_step(tok.data_ptr(), 2, logits.data_ptr(), V, st)
    torch.cuda.synchronize()
    assert pkg.status() == 0
