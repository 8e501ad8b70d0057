"""gpt2k_attention_noalloc, the attention entry point for callers that cannot
allocate device memory at call time, against gpt2k_attention (which takes its
mask scratch from a caller workspace).

Both entry points run the same kernels on the same inputs, so their outputs
must be identical bit for bit; a stale byte left in the built-in scratch by an
earlier call would show up as a difference.  Two calls in a row use
different masks, for the FP32 and the tcgen05 BF16 kernels, and each output
is also held to the float64 attention with the tolerance of the kernel tests
(2e-5 FP32, 3e-2 BF16).  A shape just past the scratch limit is refused with
a message.  Collected last, and self-contained so it also passes alone in a
fresh process."""
import pytest

from helpers import attention_ref, load_pkg

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
        assert torch.equal(got, ref), (call, (got.double() - ref.double()).abs().max().item())
        want = attention_ref(torch, qkv, mask, B, S, H)
        err = (got.double() - want).abs().max().item()
        assert err <= (2e-5 if dtype == pkg.DTYPE_F32 else 3e-2), (call, err)


def test_noalloc_rejects_shapes_past_its_scratch(torch):
    """B=4200 x S=1000 needs 256 + 4*4200 + 4200*1000 = 4,217,056 scratch bytes, just over the 4 MiB
    array.  Every buffer is sized for that shape, so if the size check ever failed the call would
    compute an attention into valid memory rather than touch memory it does not own through these
    arguments."""
    B, S, H = 4200, 1000, 1
    assert pkg.k_attention_workspace_bytes(B, S) == 4_217_056 > 4 << 20
    qkv = torch.zeros(B * S, 3 * H * 64, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros(B * S, H * 64, dtype=torch.bfloat16, device="cuda")
    mask = torch.ones(B, S, dtype=torch.int64, device="cuda")
    with pytest.raises(pkg.Gpt2Error, match="built-in array"):
        pkg.k_attention_noalloc(qkv.data_ptr(), mask.data_ptr(), o.data_ptr(), B, S, H, pkg.DTYPE_BF16,
                                torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert not o.any()  # nothing ran
