"""Weight-only FP8 configuration (GPT-2 XL shape: d 1600, 25 heads of 64,
MLP 6400; E4M3 Conv1D weights with per-output-channel scales, BF16
activations, tied BF16 lm_head) on the GPU, through the C ABI.

Two comparisons with the oracle on the same inputs (helpers.top5_check):
  * against the oracle run on the FP8-dequantized weights, which isolates the
    kernels: every logit within FP8_DEQ_MAX_REL of max |logit|, top-5 identity
    at every position checkable under the stated bound BF16_TOP5_BOUND_REL,
    and floors on the checkable fraction, top-1 agreement and top-5 overlap;
  * against the oracle on the original FP32 weights (the reference's own
    computation, quantization error included): FP8_F32_MAX_REL of max |logit|
    and floors on top-1 agreement and top-5 overlap (the quantized model is a
    different model, so top-5 identity is not required here)."""
import numpy as np
import pytest

from helpers import BF16_TOP5_BOUND_REL, FP8_DEQ_MAX_REL, FP8_F32_MAX_REL, load_oracle, load_pkg, shape_to_cfg, top5_check

pytestmark = pytest.mark.gpu
pkg = load_pkg()
O = load_oracle()


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    t.cuda.set_device(0)
    return t


def _run(shape, seed, B, S, masked):
    blob = O.seeded_blob(shape, seed, 1)
    ids = O.token_ids(B, S, seed, shape.vocab_size)
    mask = np.ones_like(ids)
    if masked and B > 1:
        mask[1, :9] = 0
    O.set_loop_threads(8)
    ref_q = O.forward(shape, O.fp8_dequantized_blob(shape, blob), ids, mask)
    ref_f = O.forward(shape, blob, ids, mask)
    O.set_loop_threads(1)
    pkg.init(shape_to_cfg(pkg, shape, pkg.DTYPE_FP8W), 0)
    pkg.load_weights(blob)
    got = pkg.gpt2_decoder(ids, mask)
    rows = np.cumsum(mask != 0, axis=1) > 0
    return ref_q[rows], ref_f[rows], got[rows]


def test_fp8w_xl_shape_two_layers(torch):
    # calibration on a B200: vs dequantized max rel 6.8e-3, checkable 5.9 %, top-1 0.982, overlap 4.92;
    # vs FP32 weights max rel 6.7e-2, top-1 0.862, overlap 4.46
    shape = O.ModelShape(n_layer=2, n_embd=1600, n_head=25, n_inner=6400)
    ref_q, ref_f, got = _run(shape, 4321, 2, 200, True)
    top5_check("fp8w XL-shape L2 vs oracle on dequantized weights", ref_q, got, max_rel=FP8_DEQ_MAX_REL,
               bound_rel=BF16_TOP5_BOUND_REL, min_checked=0.03, min_top1=0.95, min_overlap=4.85)
    top5_check("fp8w XL-shape L2 vs oracle on FP32 weights", ref_f, got, max_rel=FP8_F32_MAX_REL, min_top1=0.8,
               min_overlap=4.3)


def test_fp8w_gpt2_xl_48_layers(torch):
    """The FP8-weight workload's model (GPT-2 XL shape, 48 layers) on two sequences of 256 tokens.
    Calibration on one sequence of 128 tokens: vs dequantized max rel 1.7e-2, checkable 1.6 %, top-1
    0.961, overlap 4.82; vs FP32 weights max rel 9.7e-2, top-1 0.695, overlap 3.93."""
    ref_q, ref_f, got = _run(O.GPT2_XL, 2024, 2, 256, False)
    top5_check("fp8w GPT-2 XL vs oracle on dequantized weights", ref_q, got, max_rel=FP8_DEQ_MAX_REL,
               bound_rel=BF16_TOP5_BOUND_REL, min_checked=0.01, min_top1=0.93, min_overlap=4.7)
    top5_check("fp8w GPT-2 XL vs oracle on FP32 weights", ref_f, got, max_rel=FP8_F32_MAX_REL, min_top1=0.6,
               min_overlap=3.7)
    pkg.shutdown()


@pytest.mark.parametrize("B,S", [(4, 3), (2, 5)])
def test_fp8w_few_tokens_tensor_core_products(torch, B, S):
    """Forwards of 8-16 tokens run their products on the tensor-core GEMV with the FP8 weights'
    per-channel scales in its epilogue (K = 1600 split 5 ways over a cluster; the 6400-deep MLP
    projection falls back to the SIMT GEMV).  Too few positions for fraction floors: every logit
    within FP8_DEQ_MAX_REL of the oracle on the dequantized weights, top-5 identity wherever the
    stated bound makes it checkable."""
    shape = O.ModelShape(n_layer=2, n_embd=1600, n_head=25, n_inner=6400)
    ref_q, _, got = _run(shape, 77 + B, B, S, True)
    top5_check(f"fp8w XL-shape L2 B{B}xS{S} vs oracle on dequantized weights", ref_q, got, max_rel=FP8_DEQ_MAX_REL,
               bound_rel=BF16_TOP5_BOUND_REL)
