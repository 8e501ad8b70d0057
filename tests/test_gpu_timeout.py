"""The kernels' bounded-wait error path, exercised on the GPU without a fault.

Every mbarrier wait in the tcgen05 kernels gives up after a limit (2 s); the
kernel then records status 2 in its status word, stops issuing, waits for the
copies and MMAs it issued, frees its tensor memory and returns.  The hook
gpt2k_test_gemm_withheld_load makes one wait run out for real: CTA 0's TMA
producer never fills its first stage, so CTA 0's MMA thread waits for data
that never comes.  Nothing faults, traps or hangs: the test expects status 2
after about the wait limit, then a correct GEMM and a correct forward in the
same CUDA context.  The reference has no error path to compare with
(src/gpt/gpt2_call.cpp:42-46 checks cuInit only)."""
import time

import numpy as np
import pytest

from helpers import load_oracle, load_pkg, shape_to_cfg

pytestmark = pytest.mark.gpu
pkg = load_pkg()
O = load_oracle()


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    t.cuda.set_device(0)
    return t


def test_withheld_copy_times_out_unwinds_and_leaves_the_context_usable(torch):
    M, N, K = 1024, 1024, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    C = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pkg.k_test_gemm_withheld_load(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, status.data_ptr(), st)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) == 2  # a barrier wait timed out
    assert 1.0 <= waited < 30.0, waited  # the 2 s limit ran out once, then every role unwound

    # The context is intact: the same product through the regular entry point is right ...
    C2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    pkg.k_gemm_bf16(A.data_ptr(), B.data_ptr(), C2.data_ptr(), M, N, K, N, 0, None, None, pkg.EPI_NONE, 128, st)
    torch.cuda.synchronize()
    want = A.double() @ B.double().T
    assert (C2.double() - want).abs().max().item() <= 2e-2 * want.abs().max().item()

    # ... and so is a whole forward (tcgen05 GEMMs and attention allocate tensor memory again).
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 5, 0)
    pkg.init(shape_to_cfg(pkg, shape, pkg.DTYPE_BF16), 0)
    pkg.load_weights(blob)
    ids = O.token_ids(2, 64, 5, shape.vocab_size)
    got = pkg.gpt2_decoder(ids)
    assert pkg.status() == 0
    ref = O.forward(shape, blob, ids)
    assert np.abs(got - ref).max() <= 0.015 * np.abs(ref).max()
