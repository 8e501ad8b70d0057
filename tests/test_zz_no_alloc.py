"""gpt2k_attention_noalloc, the attention entry point for callers that cannot
allocate device memory at call time, against gpt2k_attention (which takes its
mask scratch from a caller workspace): identical outputs on two calls in a row
with different masks (the built-in scratch keeps the previous call's bytes),
for the FP32 and the tcgen05 BF16 kernels, and a clear error past the size
limit.  Collected last, and self-contained so it also passes alone in a fresh
process."""
import pytest

from helpers import load_pkg

pytestmark = pytest.mark.gpu
pkg = load_pkg()


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    t.cuda.set_device(0)
    return t


@pytest.mark.parametrize("dtype", [pkg.DTYPE_F32, pkg.DTYPE_BF16])
def test_noalloc_matches_workspace_entry_point(torch, dtype):
    B, S, H = 3, 300, 4
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(11)
    for call in range(2):
        qkv = torch.randn(B * S, 3 * H * 64, device="cuda", generator=g)
        if dtype == pkg.DTYPE_BF16:
            qkv = qkv.bfloat16()
        mask = torch.ones(B, S, dtype=torch.int64, device="cuda")
        if call == 0:
            mask[0, :7] = 0          # left padding
            mask[1, 100:150] = 0     # a hole
            mask[2, :] = 0           # nothing attendable
        else:
            mask[1, :40] = 0
            mask[2, -3:] = 0
        ref = torch.full((B * S, H * 64), 5.0, device="cuda", dtype=qkv.dtype)
        got = torch.full_like(ref, -5.0)
        ws = torch.empty(pkg.k_attention_workspace_bytes(B, S), dtype=torch.uint8, device="cuda")
        pkg.k_attention(qkv.data_ptr(), mask.data_ptr(), ref.data_ptr(), B, S, H, dtype, ws.data_ptr(), st)
        pkg.k_attention_noalloc(qkv.data_ptr(), mask.data_ptr(), got.data_ptr(), B, S, H, dtype, st)
        torch.cuda.synchronize()
        err = (got.double() - ref.double()).abs().max().item()
        assert err <= (2e-5 if dtype == pkg.DTYPE_F32 else 3e-2), (call, err)
        assert torch.isfinite(got.float()).all()


def test_noalloc_rejects_shapes_past_its_scratch(torch):
    B, S, H = 8192, 1024, 1  # 8 Mi key bytes > the 4 MiB array
    mask = torch.ones(1, dtype=torch.int64, device="cuda")
    with pytest.raises(pkg.Gpt2Error, match="built-in array"):
        pkg.k_attention_noalloc(0, mask.data_ptr(), 0, B, S, H, pkg.DTYPE_F32,
                                torch.cuda.current_stream().cuda_stream)
