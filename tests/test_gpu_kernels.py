"""Kernel-level parity on the GPU through the C ABI (gpt2k_* entry points).

FP32 kernels are held to FP32 rounding against float64 references; BF16
kernels to bf16 output rounding (the products of bf16 inputs are exact in
FP32, so only the accumulation order and the final rounding differ)."""
import numpy as np
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


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def _epi_ref(torch, acc, bias, resid, epi):
    if epi == pkg.EPI_NONE:
        return acc
    v = acc + bias.double()
    if epi == pkg.EPI_BIAS_GELU:
        v = 0.5 * v * (1.0 + torch.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))
    if epi == pkg.EPI_BIAS_GELU_ERF:
        v = 0.5 * v * (1.0 + torch.erf(v * 0.7071067811865476))
    if epi == pkg.EPI_BIAS_RESID:
        v = resid.double() + v
    return v


@pytest.mark.parametrize("M,N,K,b_nk,epi,ldc", [
    (5, 2304, 768, 0, pkg.EPI_BIAS, 2304),
    (130, 768, 3072, 0, pkg.EPI_BIAS_RESID, 768),
    (257, 3072, 768, 0, pkg.EPI_BIAS_GELU, 3072),
    (129, 3072, 768, 1, pkg.EPI_BIAS_GELU_ERF, 3072),
    (77, 50257, 768, 1, pkg.EPI_NONE, 50257),
    (64, 1000, 128, 1, pkg.EPI_NONE, 1008),
    (130, 776, 136, 0, pkg.EPI_BIAS_RESID, 776),     # 64-wide tiles, ragged N, a half K step at the end
    # enough tiles for 128-wide tiles: ragged M, both B layouts, a half K step
    (9000, 2304, 768, 0, pkg.EPI_BIAS, 2304),
    (4500, 3072, 768, 0, pkg.EPI_BIAS_GELU, 3072),
    (9000, 1000, 136, 1, pkg.EPI_NONE, 1008),
])
def test_gemm_f32(torch, M, N, K, b_nk, epi, ldc):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = (torch.randn(N, K, device="cuda", generator=g) if b_nk else torch.randn(K, N, device="cuda", generator=g)) * 0.05
    bias = torch.randn(N, device="cuda", generator=g)
    C = torch.randn(M, ldc, device="cuda", generator=g)
    resid = C[:, :N].clone()
    pkg.k_gemm_f32(A.data_ptr(), B.data_ptr(), b_nk, C.data_ptr(), M, N, K, ldc, bias.data_ptr(), C.data_ptr(), epi,
                   _stream(torch))
    torch.cuda.synchronize()
    acc = A.double() @ (B.double().T if b_nk else B.double())
    ref = _epi_ref(torch, acc, bias, resid, epi)
    err = (C[:, :N].double() - ref).abs().max().item()
    assert err <= 2e-5 * ref.abs().max().item() + 1e-6, err


@pytest.mark.parametrize("M,N,K,epi,out_f32,bn,ldc", [
    (128, 256, 64, pkg.EPI_NONE, 0, 256, 256),
    (1000, 2304, 768, pkg.EPI_BIAS, 0, 256, 2304),
    (300, 768, 3072, pkg.EPI_BIAS_RESID, 0, 128, 768),
    (513, 3072, 768, pkg.EPI_BIAS_GELU, 0, 256, 3072),
    (513, 3072, 768, pkg.EPI_BIAS_GELU_ERF, 0, 256, 3072),
    (300, 3072, 768, pkg.EPI_BIAS_GELU_ERF, 0, 128, 3072),
    (200, 50257, 768, pkg.EPI_NONE, 1, 256, 50304),
    (200, 50257, 768, pkg.EPI_NONE, 1, 128, 50257),
    (64, 1000, 128, pkg.EPI_BIAS, 1, 128, 1000),
    (4096, 768, 768, pkg.EPI_BIAS_RESID, 0, 256, 768),
    # bn = 2: 256 x 256 tiles on CTA pairs (tcgen05.mma.cta_group::2)
    (256, 256, 64, pkg.EPI_NONE, 0, 2, 256),
    (100, 2304, 768, pkg.EPI_BIAS, 0, 2, 2304),       # the second CTA's rows all past M
    (1000, 2304, 768, pkg.EPI_BIAS, 0, 2, 2304),
    (300, 768, 3072, pkg.EPI_BIAS_RESID, 0, 2, 768),
    (513, 3072, 768, pkg.EPI_BIAS_GELU, 0, 2, 3072),
    (513, 3072, 768, pkg.EPI_BIAS_GELU_ERF, 0, 2, 3072),
    (8192, 3072, 768, pkg.EPI_BIAS_GELU, 0, 2, 3072),  # more tiles than pairs: both accumulators
    (8192, 768, 3072, pkg.EPI_BIAS_RESID, 0, 2, 768),
    (200, 50257, 768, pkg.EPI_NONE, 1, 2, 50304),
    (1000, 1000, 136, pkg.EPI_BIAS, 1, 2, 1000),        # ragged K (zero-filled) and N
    (200, 50257, 768, pkg.EPI_NONE, 1, 2, 50257),       # C not TMA-storable: single-SM kernel
])
def test_gemm_bf16_tcgen05(torch, M, N, K, epi, out_f32, bn, ldc):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    if out_f32:
        C = torch.full((M, ldc), 7.0, device="cuda")
    else:
        C = torch.randn(M, ldc, device="cuda", generator=g).bfloat16()
    resid = C[:, :N].clone()
    pkg.k_gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, ldc, out_f32, bias.data_ptr(),
                    C.data_ptr(), epi, bn, _stream(torch))
    torch.cuda.synchronize()
    acc = A.double() @ B.double().T
    ref = _epi_ref(torch, acc, bias, resid, epi)
    got = C[:, :N].double()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    if out_f32:
        assert err <= 1e-5 * scale, (err, scale)
        # padding columns past the row's last 16-byte unit are untouched (the TMA store
        # writes whole 16-byte units at the ragged edge)
        edge = (N + 3) // 4 * 4
        if ldc > edge:
            assert torch.all(C[:, edge:] == 7.0)
    else:
        assert err <= 8e-3 * scale, (err, scale)


def _row_stats(torch, x):
    """Per row and 128-column segment: (sum, sum of squares) of x's values, float32 [M, nseg, 2]."""
    M, K = x.shape
    nseg = (K + pkg.LN_SEG - 1) // pkg.LN_SEG
    xp = torch.zeros(M, nseg * pkg.LN_SEG, dtype=torch.float64, device=x.device)
    xp[:, :K] = x.double()
    xp = xp.view(M, nseg, pkg.LN_SEG)
    return torch.stack([xp.sum(-1), (xp * xp).sum(-1)], -1).float().contiguous()


def _vec_len(n):
    return (n + 255) // 256 * 256


@pytest.mark.parametrize("M,N,K,epi,out_f32,bn,ldc", [
    (1000, 2304, 768, pkg.EPI_LN_BIAS, 0, 256, 2304),
    (513, 3072, 768, pkg.EPI_LN_BIAS_GELU, 0, 2, 3072),
    (513, 3072, 768, pkg.EPI_LN_BIAS_GELU, 0, 128, 3072),
    (300, 50257, 768, pkg.EPI_LN_BIAS, 1, 2, 50304),    # the lm_head with ln_f folded in
    (200, 1000, 768, pkg.EPI_LN_BIAS, 1, 128, 1000),
    (77, 384, 1600, pkg.EPI_LN_BIAS_GELU, 0, 128, 384),  # K = 1600: a partial last segment
])
def test_gemm_layernorm_folded(torch, M, N, K, epi, out_f32, bn, ldc):
    """LN(x) @ W + bias (then gelu_new) with the LayerNorm folded into the GEMM: gain-scaled bf16
    weight, c1 / c2 vectors and row statistics, against LayerNorm then the linear layer in float64."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    # rows with their own offset and scale, as in a residual stream
    x = (torch.randn(M, K, device="cuda", generator=g) * (0.5 + torch.rand(M, 1, device="cuda", generator=g) * 3)
         + torch.randn(M, 1, device="cuda", generator=g)).bfloat16()
    gain = 1.0 + 0.2 * torch.randn(K, device="cuda", generator=g)
    shift = 0.1 * torch.randn(K, device="cuda", generator=g)
    W = 0.05 * torch.randn(K, N, device="cuda", generator=g)  # Conv1D layout [in, out]
    bias = 0.1 * torch.randn(N, device="cuda", generator=g)
    B = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
    c1 = torch.full((_vec_len(N),), 9.0, device="cuda")
    c2 = torch.full((_vec_len(N),), 9.0, device="cuda")
    pkg.k_ln_fold_pack(W.data_ptr(), 1, gain.data_ptr(), shift.data_ptr(), bias.data_ptr(), B.data_ptr(),
                       c1.data_ptr(), c2.data_ptr(), N, K, _stream(torch))
    torch.cuda.synchronize()
    assert torch.equal(B, (W.T * gain).bfloat16())
    assert torch.allclose(c1[:N].double(), B.double().sum(1), rtol=1e-6, atol=1e-5)
    assert torch.allclose(c2[:N].double(), W.double().T @ shift.double() + bias.double(), rtol=1e-6, atol=1e-5)
    assert torch.all(c1[N:] == 0) and torch.all(c2[N:] == 0)
    stats = _row_stats(torch, x)
    C = torch.zeros(M, ldc, device="cuda", dtype=torch.float32 if out_f32 else torch.bfloat16)
    eps = 1e-5
    pkg.k_gemm_bf16_ln(x.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, ldc, out_f32, None, None, epi, bn,
                       c1.data_ptr(), c2.data_ptr(), stats.data_ptr(), None, eps, _stream(torch))
    torch.cuda.synchronize()
    xd = x.double()
    mu = xd.mean(1, keepdim=True)
    var = ((xd - mu) ** 2).mean(1, keepdim=True)
    ln = (xd - mu) / torch.sqrt(var + eps) * gain.double() + shift.double()
    ref = ln @ W.double() + bias.double()
    if epi == pkg.EPI_LN_BIAS_GELU:
        ref = 0.5 * ref * (1.0 + torch.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
    got = C[:, :N].double()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    # bf16 weights (W * gain rounded) and, for bf16 C, the output rounding
    assert err <= 8e-3 * scale, (err, scale)
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel <= 4e-3, rel


@pytest.mark.parametrize("M,N,K,bn", [(1000, 768, 768, 256), (513, 768, 3072, 2), (300, 1000, 512, 128),
                                      (8192, 768, 3072, 2)])
def test_gemm_residual_row_stats(torch, M, N, K, bn):
    """EPI_BIAS_RESID_STATS: C = resid + A @ B^T + bias, and the per-segment sums of the stored bf16 C."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    Bw = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    C = (torch.randn(M, N, device="cuda", generator=g) * 3).bfloat16()
    resid = C.clone()
    nseg = (N + pkg.LN_SEG - 1) // pkg.LN_SEG
    stats = torch.full((M, nseg, 2), 7.0, device="cuda")
    pkg.k_gemm_bf16_ln(A.data_ptr(), Bw.data_ptr(), C.data_ptr(), M, N, K, N, 0, bias.data_ptr(), C.data_ptr(),
                       pkg.EPI_BIAS_RESID_STATS, bn, None, None, None, stats.data_ptr(), 1e-5, _stream(torch))
    torch.cuda.synchronize()
    ref = resid.double() + A.double() @ Bw.double().T + bias.double()
    assert (C.double() - ref).abs().max().item() <= 8e-3 * ref.abs().max().item()
    want = _row_stats(torch, C).double()
    assert torch.allclose(stats.double(), want, rtol=2e-5, atol=1e-3), (stats - want).abs().max()


@pytest.mark.parametrize("T,d,dtype", [(1000, 768, 0), (33, 1600, 0), (1000, 768, 1), (5, 128, 1), (7, 1600, 1)])
def test_layernorm(torch, T, d, dtype):
    g = torch.Generator(device="cuda").manual_seed(T + d)
    x = torch.randn(T, d, device="cuda", generator=g) * 3 + 0.5
    gain = 1 + 0.1 * torch.randn(d, device="cuda", generator=g)
    shift = 0.1 * torch.randn(d, device="cuda", generator=g)
    if dtype == 1:
        x = x.bfloat16()
    y = torch.empty_like(x)
    pkg.k_layernorm(x.data_ptr(), gain.data_ptr(), shift.data_ptr(), y.data_ptr(), T, d, 1e-5, dtype, _stream(torch))
    torch.cuda.synchronize()
    ref = torch.nn.functional.layer_norm(x.double(), (d,), gain.double(), shift.double(), 1e-5)
    err = (y.double() - ref).abs().max().item()
    assert err <= (1e-5 if dtype == 0 else 2e-2 * ref.abs().max().item()), err


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("B,S,H,masked", [(2, 1, 12, False), (3, 77, 2, True), (1, 1024, 12, False),
                                          (2, 128, 2, True), (2, 200, 12, True), (2, 257, 3, False),
                                          (4, 384, 2, True), (1, 1000, 12, False), (3, 64, 2, True),
                                          (2, 65, 12, False)])
def test_attention(torch, dtype, B, S, H, masked):
    """dtype 0: FP32 SIMT; 1: tcgen05 BF16."""
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S)
    qkv = torch.randn(B * S, 3 * H * 64, device="cuda", generator=g)
    mask = None
    if masked:
        mask = torch.ones(B, S, dtype=torch.int64, device="cuda")
        mask[0, : min(5, S)] = 0                 # left padding
        if B > 1:
            mask[1, S // 3: S // 2] = 0          # a hole
            mask[1, -1] = 0                      # right padding
        if B > 2:
            mask[2, :] = 0                       # nothing attendable
    if dtype >= 1:
        qkv = qkv.bfloat16()
    o = torch.full((B * S, H * 64), 3.0, device="cuda", dtype=qkv.dtype)
    ws = torch.empty(pkg.k_attention_workspace_bytes(B, S), dtype=torch.uint8, device="cuda")
    pkg.k_attention(qkv.data_ptr(), mask.data_ptr() if mask is not None else None, o.data_ptr(), B, S, H,
                    dtype, ws.data_ptr(), _stream(torch))
    torch.cuda.synchronize()
    ref = attention_ref(torch, qkv, mask, B, S, H)
    err = (o.double() - ref).abs().max().item()
    assert err <= (2e-5 if dtype == 0 else 3e-2), err
    assert torch.isfinite(o.float()).all()


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("B,S,H,mask_kind", [(2, 1, 12, None), (3, 77, 2, "mixed"), (1, 512, 12, None),
                                             (4, 512, 2, "right"), (3, 300, 12, "mixed"), (2, 129, 3, "right"),
                                             (5, 384, 2, "right")])
def test_attention_non_causal(torch, dtype, B, S, H, mask_kind):
    """The encoder (BERT) form: every unmasked key of the sequence; right padding (lengths ending
    inside, on and past 128-key tiles, so key tiles past the last valid key are skipped), holes,
    left padding and a sequence with no unmasked key."""
    g = torch.Generator(device="cuda").manual_seed(B * 7919 + S)
    qkv = torch.randn(B * S, 3 * H * 64, device="cuda", generator=g)
    mask = None
    if mask_kind == "right":
        lens = [S, max(1, S // 2), 64, 128, 129, 1][:B]
        mask = torch.zeros(B, S, dtype=torch.int64, device="cuda")
        for b, n in enumerate(lens):
            mask[b, :min(n, S)] = 1
    elif mask_kind == "mixed":
        mask = torch.ones(B, S, dtype=torch.int64, device="cuda")
        mask[0, : min(5, S)] = 0
        if B > 1:
            mask[1, S // 3: S // 2] = 0
        if B > 2:
            mask[2, :] = 0
    if dtype >= 1:
        qkv = qkv.bfloat16()
    o = torch.full((B * S, H * 64), 3.0, device="cuda", dtype=qkv.dtype)
    ws = torch.empty(pkg.k_attention_ex_workspace_bytes(B, S), dtype=torch.uint8, device="cuda")
    pkg.k_attention_ex(qkv.data_ptr(), mask.data_ptr() if mask is not None else None, o.data_ptr(), B, S, H, dtype, 0,
                       ws.data_ptr(), _stream(torch))
    torch.cuda.synchronize()
    ref = attention_ref(torch, qkv, mask, B, S, H, causal=False)
    err = (o.double() - ref).abs().max().item()
    assert err <= (2e-5 if dtype == 0 else 3e-2), err
    # causal = 1 through the same entry point equals gpt2k_attention
    o2 = torch.full_like(o, 3.0)
    pkg.k_attention_ex(qkv.data_ptr(), mask.data_ptr() if mask is not None else None, o2.data_ptr(), B, S, H, dtype,
                       1, ws.data_ptr(), _stream(torch))
    torch.cuda.synchronize()
    ref_c = attention_ref(torch, qkv, mask, B, S, H, causal=True)
    assert (o2.double() - ref_c).abs().max().item() <= (2e-5 if dtype == 0 else 3e-2)


@pytest.mark.parametrize("dtype", [0, 1])
def test_embed_and_bad_ids(torch, dtype):
    V, P, d, S = 1000, 64, 128, 10
    g = torch.Generator(device="cuda").manual_seed(5)
    wte = torch.randn(V, d, device="cuda", generator=g)
    wpe = torch.randn(P, d, device="cuda", generator=g)
    if dtype == 1:
        wte, wpe = wte.bfloat16(), wpe.bfloat16()
    ids = torch.randint(0, V, (2, S), device="cuda", generator=g)
    ids[1, 3] = V  # out of range
    x = torch.empty(2 * S, d, device="cuda", dtype=wte.dtype)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg.k_embed(ids.data_ptr(), wte.data_ptr(), wpe.data_ptr(), x.data_ptr(), 2 * S, S, d, V, dtype,
                status.data_ptr(), _stream(torch))
    torch.cuda.synchronize()
    assert status.item() == 1
    ref = wte.double()[ids.clamp(max=V - 1)].reshape(2 * S, d) + wpe.double()[torch.arange(S, device="cuda").repeat(2)]
    good = torch.ones(2 * S, dtype=torch.bool, device="cuda")
    good[S + 3] = False
    err = (x.double()[good] - ref[good]).abs().max().item()
    assert err <= (1e-6 if dtype == 0 else 3e-2), err
    assert torch.all(x[S + 3].double() == wpe.double()[3])


@pytest.mark.parametrize("M,N,K,transB,where", [(77, 50, 33, 111, "host"), (128, 256, 64, 111, "device"),
                                                (5, 2304, 768, 111, "host"), (40, 100, 17, 112, "device"),
                                                (64, 1000, 128, 112, "host")])
def test_blas_sgemm_lowering_call(torch, M, N, K, transB, where):
    """gpt2_blas_sgemm with the argument list a BLAS lowering of linalg.matmul emits
    (lib/ConvertMatMulToBlas.cpp:84-160: RowMajor, NoTrans, alpha 1, beta 0, lda K, ldb N, ldc N),
    on host or device operands, shapes the SIMT kernel needs padded for included."""
    import ctypes
    rng = np.random.default_rng(M * 131 + N)
    A = rng.standard_normal((M, K), dtype=np.float32)
    Bm = rng.standard_normal((N, K) if transB == 112 else (K, N), dtype=np.float32)
    ref = A.astype(np.float64) @ (Bm.T if transB == 112 else Bm).astype(np.float64)
    lib = pkg.lib()
    ldb = K if transB == 112 else N
    if where == "host":
        C = np.full((M, N), 7.0, dtype=np.float32)
        rc = lib.gpt2_blas_sgemm(101, 111, transB, M, N, K, 1.0, A.ctypes.data, K, Bm.ctypes.data, ldb, 0.0,
                                 C.ctypes.data, N)
        got = C
    else:
        dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(Bm).cuda()
        dC = torch.full((M, N), 7.0, device="cuda")
        rc = lib.gpt2_blas_sgemm(101, 111, transB, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), ldb, 0.0,
                                 dC.data_ptr(), N)
        got = dC.cpu().numpy()
    assert rc == 0, pkg.last_error()
    assert np.abs(got - ref).max() <= 2e-5 * np.abs(ref).max() + 1e-5
    # calls the lowering never emits are refused, not computed
    assert lib.gpt2_blas_sgemm(101, 111, 111, M, N, K, 2.0, A.ctypes.data, K, A.ctypes.data, N, 0.0,
                               A.ctypes.data, N) == pkg_einval()


def pkg_einval():
    return -1


# The few-token / decode products (gpt2k_gemv_bf16): the SIMT kernel (impl 0)
# and the tensor-core kernel (impl 1, weights as the 128-row MMA operand, K
# split over a thread-block cluster) against a float64 reference.  A
# LayerNorm'd row enters the tensor-core kernel as two bf16 operands (hi and
# lo), so both kernels multiply FP32 rows by bf16 weights and are held to the
# bf16 rounding of the output: 1 % of the largest |y|.
@pytest.mark.parametrize("M,N,K,epi,ln,out_f32", [
    (1, 768, 768, pkg.EPI_BIAS, True, 0),             # one row (B = 1 decode)
    (5, 2304, 768, pkg.EPI_BIAS, True, 0),            # QKV with ln_1, few rows
    (16, 3072, 768, pkg.EPI_BIAS_GELU, True, 0),      # MLP fc with ln_2
    (16, 768, 768, pkg.EPI_BIAS_RESID, False, 0),     # attention out-proj (6 weight tiles: K split 6 ways)
    (16, 768, 3072, pkg.EPI_BIAS_RESID, False, 0),    # MLP proj (K = 3072: split 8 ways)
    (3, 3072, 768, pkg.EPI_BIAS_GELU_ERF, False, 0),  # BERT's GELU (the SIMT kernel has it without a LayerNorm)
    (7, 1000, 128, pkg.EPI_NONE, False, 0),           # ragged N, two k-steps
    (16, 50257, 768, pkg.EPI_NONE, True, 1),          # lm_head with ln_f, FP32 logits
])
def test_gemv_bf16_both_kernels(torch, M, N, K, epi, ln, out_f32):
    g = torch.Generator(device="cuda").manual_seed(M * 131 + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    gain = (1.0 + 0.1 * torch.randn(K, device="cuda", generator=g)).float()
    shift = (0.1 * torch.randn(K, device="cuda", generator=g)).float()
    resid0 = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    xd = x.double()
    if ln:
        mu = xd.mean(1, keepdim=True)
        var = ((xd - mu) ** 2).mean(1, keepdim=True)
        xd = (xd - mu) / torch.sqrt(var + 1e-5) * gain.double() + shift.double()
    ref = _epi_ref(torch, xd @ W.double().T, bias, resid0, epi)
    scale = ref.abs().max().item()
    outs = []
    for impl in (0, 1, 1):
        y = resid0.clone() if not out_f32 else torch.zeros(M, N, device="cuda")
        pkg.k_gemv_bf16(x.data_ptr(), W.data_ptr(), y.data_ptr(), M, N, K, N,
                        bias.data_ptr() if epi != pkg.EPI_NONE else None,
                        y.data_ptr() if epi == pkg.EPI_BIAS_RESID else None, epi,
                        gain.data_ptr() if ln else None, shift.data_ptr() if ln else None, 1e-5,
                        out_f32, impl, _stream(torch))
        torch.cuda.synchronize()
        err = (y.double() - ref).abs().max().item()
        assert err <= 1e-2 * scale, (impl, err, scale)
        outs.append(y)
    # The split-K partial sums meet in a fixed order: repeated runs agree bit for bit.
    assert torch.equal(outs[1], outs[2])


def test_gemv_bf16_rejects_what_the_tensor_core_kernel_cannot_do(torch):
    x = torch.zeros(4, 136, device="cuda", dtype=torch.bfloat16)
    W = torch.zeros(64, 136, device="cuda", dtype=torch.bfloat16)
    y = torch.zeros(4, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(pkg.Gpt2Error, match="multiple of 64"):
        pkg.k_gemv_bf16(x.data_ptr(), W.data_ptr(), y.data_ptr(), 4, 64, 136, 64, impl=1, stream=_stream(torch))
    with pytest.raises(pkg.Gpt2Error, match="bad operands"):
        pkg.k_gemv_bf16(x.data_ptr(), W.data_ptr(), y.data_ptr(), 17, 64, 136, 64, impl=0, stream=_stream(torch))
