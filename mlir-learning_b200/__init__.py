"""Python host mirror of libgpt2_b200.so (the C ABI in include/gpt2_b200.h).

The reference calls its compiled GPT-2 through the memref C ABI from C++
(src/gpt/gpt2_call.cpp:31-64) and defines the operator in Python as
GPT2Wrapper.forward(input_ids, attention_mask) -> logits
(src/gpt/lower_gpt_model.py:20-50).  This module binds the same entry points
with ctypes:

  * `gpt2_decoder(ids, mask)` / `ciface_gpt2_decoder(ids, mask)`: the two
    drop-in symbols, numpy int64 [B, S] in, FP32 logits [B, S, V] out;
  * `GPT2Decoder(...).forward(input_ids, attention_mask)`: the wrapper's
    operator shape over the same library;
  * device-side entry points (`forward_device`, kernel-level `k_*`) taking raw
    device pointers, used by the benchmark and the parity tests.

There is no CPU fallback: every call goes to the CUDA library, and importing
fails loudly when the library has not been built.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgpt2_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "gpt2_b200.h")
BERT_HEADER = os.path.join(os.path.dirname(HERE), "include", "bert_b200.h")

DTYPE_F32, DTYPE_BF16, DTYPE_FP8W = 0, 1, 2
EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESID, EPI_BIAS_GELU_ERF = 0, 1, 2, 3, 4
EPI_LN_BIAS, EPI_LN_BIAS_GELU, EPI_BIAS_RESID_STATS = 5, 6, 7
LN_SEG = 128  # columns per row-statistics segment of the folded LayerNorm
STATUS_NAMES = {0: "ok", 1: "token id out of range", 2: "barrier wait timed out", 3: "bad launch"}


class Gpt2Config(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int32),
        ("n_embd", ctypes.c_int32),
        ("n_head", ctypes.c_int32),
        ("n_inner", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("n_positions", ctypes.c_int32),
        ("layer_norm_eps", ctypes.c_float),
        ("dtype", ctypes.c_int32),
    ]


def gpt2_small(dtype: int = DTYPE_F32) -> Gpt2Config:
    """GPT-2 124M: 12 layers, d 768, 12 heads of 64, MLP 3072, vocab 50257, ctx 1024."""
    return Gpt2Config(12, 768, 12, 3072, 50257, 1024, 1e-5, dtype)


class MemRef3D(ctypes.Structure):
    _fields_ = [
        ("allocated", ctypes.POINTER(ctypes.c_float)),
        ("aligned", ctypes.POINTER(ctypes.c_float)),
        ("offset", ctypes.c_int64),
        ("sizes", ctypes.c_int64 * 3),
        ("strides", ctypes.c_int64 * 3),
    ]


class MemRef2D_i64(ctypes.Structure):
    _fields_ = [
        ("allocated", ctypes.POINTER(ctypes.c_int64)),
        ("aligned", ctypes.POINTER(ctypes.c_int64)),
        ("offset", ctypes.c_int64),
        ("sizes", ctypes.c_int64 * 2),
        ("strides", ctypes.c_int64 * 2),
    ]


class Gpt2Error(RuntimeError):
    pass


def build(verbose: bool = False) -> str:
    """Compiles libgpt2_b200.so in-tree with nvcc for sm_100a (make -C this directory)."""
    out = subprocess.run(["make", "-C", HERE, "-j8"], capture_output=True, text=True)
    if out.returncode != 0:
        raise Gpt2Error("libgpt2_b200.so build failed:\n" + out.stdout[-4000:] + out.stderr[-4000:])
    if verbose:
        print(out.stdout)
    return LIB_PATH


_lib = None
_libc = ctypes.CDLL(None)
_libc.free.argtypes = [ctypes.c_void_p]


def lib() -> ctypes.CDLL:
    """The loaded C library; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise Gpt2Error(f"{LIB_PATH} is missing: build it with __graft_entry__.build() or make -C {HERE}")
    L = ctypes.CDLL(LIB_PATH)
    P, i64, i32, vp = ctypes.POINTER, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    L.gpt2_decoder.restype = MemRef3D
    L.gpt2_decoder.argtypes = [P(i64), P(i64), i64, i64, i64, i64, i64, P(i64), P(i64), i64, i64, i64, i64, i64]
    L._mlir_ciface_gpt2_decoder.restype = None
    L._mlir_ciface_gpt2_decoder.argtypes = [P(MemRef3D), P(MemRef2D_i64), P(MemRef2D_i64)]
    L.gpt2_init.argtypes = [P(Gpt2Config), i32]
    L.gpt2_blob_floats.argtypes = [P(Gpt2Config)]
    L.gpt2_blob_floats.restype = i64
    L.gpt2_load_weights.argtypes = [vp, ctypes.c_size_t, ctypes.c_char_p]
    L.gpt2_init_seeded.argtypes = [ctypes.c_uint64, i32]
    L.gpt2_seeded_blob.argtypes = [P(Gpt2Config), ctypes.c_uint64, i32, P(ctypes.c_float)]
    L.gpt2_seeded_ids.argtypes = [P(i64), i64, ctypes.c_uint64, ctypes.c_uint32, i64]
    L.gpt2_get_config.argtypes = [P(Gpt2Config)]
    L.gpt2_fp8_quantize.argtypes = [P(ctypes.c_float), i32, i32, P(ctypes.c_uint8), P(ctypes.c_float)]
    L.gpt2_shutdown.restype = None
    L.gpt2_last_error.restype = ctypes.c_char_p
    L.gpt2_forward_device.argtypes = [vp, vp, i32, i32, vp, i64, i32, vp]
    L.gpt2_forward_host.argtypes = [P(i64), P(i64), i32, i32, P(ctypes.c_float)]
    L.gpt2_forward_launches.argtypes = [i32, i32, i32]
    L.gpt2_profile_end.argtypes = [P(ctypes.c_double), P(i64), i32]
    L.gpt2_safetensors_to_blob.argtypes = [ctypes.c_char_p, P(Gpt2Config), P(ctypes.c_float)]
    L.gpt2_load_safetensors.argtypes = [ctypes.c_char_p]
    L.gpt2_blas_sgemm.argtypes = [i32, i32, i32, i32, i32, i32, ctypes.c_float, vp, i32, vp, i32, ctypes.c_float,
                                  vp, i32]
    L.gpt2_kv_reserve.argtypes = [i32, i32]
    L.gpt2_prefill.argtypes = [vp, i32, i32, vp, i64, vp]
    L.gpt2_decode_step.argtypes = [vp, i32, vp, i64, vp]
    L.gpt2_generate.argtypes = [P(i64), i32, i32, i32, P(i64)]
    L.gpt2k_gemm_f32.argtypes = [vp, vp, i32, vp, i32, i32, i32, i32, vp, vp, i32, vp]
    L.gpt2k_gemm_bf16.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp]
    L.gpt2k_gemv_bf16.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, vp, i32, vp, vp, ctypes.c_float, i32, i32, vp]
    L.gpt2k_test_gemm_withheld_load.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp]
    L.gpt2k_gemm_bf16_ln.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, vp, vp, vp,
                                     ctypes.c_float, vp]
    L.gpt2k_ln_fold_pack.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp, i32, i32, vp]
    L.gpt2k_ffma_peak.argtypes = [P(ctypes.c_float), vp]
    L.gpt2k_layernorm.argtypes = [vp, vp, vp, vp, i32, i32, ctypes.c_float, i32, vp]
    L.gpt2k_attention_workspace_bytes.argtypes = [i32, i32]
    L.gpt2k_attention_workspace_bytes.restype = ctypes.c_size_t
    L.gpt2k_attention.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, vp]
    L.gpt2k_attention_noalloc.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp]
    L.gpt2k_attention_ex_workspace_bytes.argtypes = [i32, i32]
    L.gpt2k_attention_ex_workspace_bytes.restype = ctypes.c_size_t
    L.gpt2k_attention_ex.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp, vp]
    L.gpt2k_embed.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp]
    _lib = L
    return L


def last_error() -> str:
    return lib().gpt2_last_error().decode()


def _check(rc: int, what: str) -> int:
    if rc < 0:
        raise Gpt2Error(f"{what} failed ({rc}): {last_error()}")
    return rc


def declared_functions(headers: tuple[str, ...] = (HEADER, BERT_HEADER)) -> list[str]:
    """Names of the functions include/gpt2_b200.h and include/bert_b200.h declare."""
    import re
    names = set()
    for h in headers:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = "\n".join(line for line in text.splitlines() if not line.lstrip().startswith("#"))
        names |= set(re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text))
    return sorted(names)


# ---------------------------------------------------------------------------
# model management
# ---------------------------------------------------------------------------
def init(cfg: Gpt2Config, device: int = -1) -> None:
    _check(lib().gpt2_init(ctypes.byref(cfg), device), "gpt2_init")


def get_config() -> Gpt2Config:
    cfg = Gpt2Config()
    _check(lib().gpt2_get_config(ctypes.byref(cfg)), "gpt2_get_config")
    return cfg


def blob_floats(cfg: Gpt2Config) -> int:
    return _check(lib().gpt2_blob_floats(ctypes.byref(cfg)), "gpt2_blob_floats")


def seeded_blob(cfg: Gpt2Config, seed: int, init_mode: int = 0) -> np.ndarray:
    out = np.empty(blob_floats(cfg), dtype=np.float32)
    _check(lib().gpt2_seeded_blob(ctypes.byref(cfg), seed, init_mode,
                                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "gpt2_seeded_blob")
    return out


def seeded_ids(B: int, S: int, seed: int, vocab: int, stream: int = 0x10000) -> np.ndarray:
    out = np.empty(B * S, dtype=np.int64)
    _check(lib().gpt2_seeded_ids(out.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), B * S, seed, stream, vocab),
           "gpt2_seeded_ids")
    return out.reshape(B, S)


def fp8_quantize(w: np.ndarray):
    """Conv1D weight w [K, N] -> (q [N, K] E4M3 codes, scale [N]) as the model quantizes it."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    K, N = w.shape
    q = np.empty((N, K), dtype=np.uint8)
    sc = np.empty(N, dtype=np.float32)
    _check(lib().gpt2_fp8_quantize(w.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), K, N,
                                   q.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                   sc.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "gpt2_fp8_quantize")
    return q, sc


def gpt2_xl(dtype: int = DTYPE_FP8W) -> Gpt2Config:
    """GPT-2 XL shape: 48 layers, d 1600, 25 heads of 64, MLP 6400, vocab 50257, ctx 1024."""
    return Gpt2Config(48, 1600, 25, 6400, 50257, 1024, 1e-5, dtype)


def load_weights(blob: np.ndarray, manifest: str | None = None) -> None:
    blob = np.ascontiguousarray(blob, dtype=np.float32)
    _check(lib().gpt2_load_weights(blob.ctypes.data, blob.nbytes, manifest.encode() if manifest else None),
           "gpt2_load_weights")


def safetensors_to_blob(path: str, cfg: Gpt2Config) -> np.ndarray:
    """The canonical FP32 blob of an HF GPT-2 safetensors checkpoint (no GPU needed)."""
    out = np.empty(blob_floats(cfg), dtype=np.float32)
    _check(lib().gpt2_safetensors_to_blob(os.fsencode(path), ctypes.byref(cfg),
                                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "gpt2_safetensors_to_blob")
    return out


def load_safetensors(path: str) -> None:
    _check(lib().gpt2_load_safetensors(os.fsencode(path)), "gpt2_load_safetensors")


def init_seeded(seed: int, init_mode: int = 0) -> None:
    _check(lib().gpt2_init_seeded(seed, init_mode), "gpt2_init_seeded")


def shutdown() -> None:
    lib().gpt2_shutdown()


def status() -> int:
    return lib().gpt2_status()


def forward_launches(B: int, S: int, has_mask: bool) -> int:
    return _check(lib().gpt2_forward_launches(B, S, int(has_mask)), "gpt2_forward_launches")


# ---------------------------------------------------------------------------
# forward entry points
# ---------------------------------------------------------------------------
def _as_i64(a) -> np.ndarray:
    a = np.asarray(a, dtype=np.int64)
    if a.ndim != 2:
        raise ValueError("ids and mask are [B, S]")
    return a


def _take_memref(m: MemRef3D) -> np.ndarray:
    if not m.allocated:
        raise Gpt2Error(f"gpt2_decoder failed: {last_error()}")
    n = m.sizes[0] * m.sizes[1] * m.sizes[2]
    view = np.ctypeslib.as_array(m.aligned, shape=(n,))
    out = view.reshape(m.sizes[0], m.sizes[1], m.sizes[2]).copy()
    _libc.free(ctypes.cast(m.allocated, ctypes.c_void_p))
    return out


def gpt2_decoder(input_ids, attention_mask=None) -> np.ndarray:
    """Calls the decomposed-memref `gpt2_decoder` exactly as src/gpt/gpt2_call.cpp:62-64 does
    (strides honoured, malloc'd result freed after copying)."""
    ids = _as_i64(input_ids)
    mask = _as_i64(attention_mask) if attention_mask is not None else np.ones_like(ids)
    P = ctypes.POINTER(ctypes.c_int64)
    ip, mp = ids.ctypes.data_as(P), mask.ctypes.data_as(P)
    isz, msz = ids.itemsize, mask.itemsize
    m = lib().gpt2_decoder(ip, ip, 0, ids.shape[0], ids.shape[1], ids.strides[0] // isz, ids.strides[1] // isz,
                           mp, mp, 0, mask.shape[0], mask.shape[1], mask.strides[0] // msz, mask.strides[1] // msz)
    return _take_memref(m)


def ciface_gpt2_decoder(input_ids, attention_mask=None) -> np.ndarray:
    """Calls `_mlir_ciface_gpt2_decoder` (descriptor pointers, result out-parameter)."""
    ids = _as_i64(input_ids)
    mask = _as_i64(attention_mask) if attention_mask is not None else np.ones_like(ids)

    def desc(a):
        p = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
        return MemRef2D_i64(p, p, 0, (ctypes.c_int64 * 2)(*a.shape),
                            (ctypes.c_int64 * 2)(a.strides[0] // a.itemsize, a.strides[1] // a.itemsize))

    res = MemRef3D()
    di, dm = desc(ids), desc(mask)
    lib()._mlir_ciface_gpt2_decoder(ctypes.byref(res), ctypes.byref(di), ctypes.byref(dm))
    return _take_memref(res)


def forward_host(input_ids, attention_mask=None) -> np.ndarray:
    ids = np.ascontiguousarray(_as_i64(input_ids))
    B, S = ids.shape
    mask_p = None
    if attention_mask is not None:
        mask = np.ascontiguousarray(_as_i64(attention_mask))
        mask_p = mask.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
    vocab = get_config().vocab_size
    out = np.empty((B, S, vocab), dtype=np.float32)
    _check(lib().gpt2_forward_host(ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), mask_p, B, S,
                                   out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "gpt2_forward_host")
    return out


def forward_device(ids_ptr: int, mask_ptr: int | None, B: int, S: int, logits_ptr: int, ld_logits: int,
                   stream_ptr: int | None = None, logits_dtype: int = DTYPE_F32) -> None:
    """gpt2_forward_device: logits_dtype DTYPE_F32 (default) or DTYPE_BF16 (ld_logits in elements)."""
    _check(lib().gpt2_forward_device(ids_ptr, mask_ptr, B, S, logits_ptr, ld_logits, logits_dtype, stream_ptr),
           "gpt2_forward_device")


def kv_reserve(B: int, max_len: int) -> None:
    _check(lib().gpt2_kv_reserve(B, max_len), "gpt2_kv_reserve")


def prefill(ids_ptr: int, B: int, S: int, logits_ptr: int, ld: int, stream_ptr: int | None = None) -> None:
    _check(lib().gpt2_prefill(ids_ptr, B, S, logits_ptr, ld, stream_ptr), "gpt2_prefill")


def decode_step(tokens_ptr: int, B: int, logits_ptr: int, ld: int, stream_ptr: int | None = None) -> None:
    _check(lib().gpt2_decode_step(tokens_ptr, B, logits_ptr, ld, stream_ptr), "gpt2_decode_step")


def kv_length() -> int:
    return lib().gpt2_kv_length()


def generate(input_ids, n_new: int) -> np.ndarray:
    """Greedy continuation of each prompt row: int64 [B, n_new] (the argmax chain HF generate's greedy
    search produces, src/gpt/run_gpt.py:20-24), with a KV cache on the GPU."""
    ids = np.ascontiguousarray(_as_i64(input_ids))
    B, S = ids.shape
    out = np.empty((B, n_new), dtype=np.int64)
    P = ctypes.POINTER(ctypes.c_int64)
    _check(lib().gpt2_generate(ids.ctypes.data_as(P), B, S, n_new, out.ctypes.data_as(P)), "gpt2_generate")
    return out


KERNEL_KINDS = ["seq_info", "embed", "layernorm", "gemm_qkv", "attention", "masked_rows", "gemm_proj", "gemm_fc",
                "gemm_mproj", "lm_head"]


def profile_begin() -> None:
    _check(lib().gpt2_profile_begin(), "gpt2_profile_begin")


def profile_end() -> dict:
    """{kind: (total ms, launches)} of the launches since profile_begin()."""
    n = len(KERNEL_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int64 * n)()
    _check(lib().gpt2_profile_end(ms, cnt, n), "gpt2_profile_end")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(KERNEL_KINDS)}


class GPT2Decoder:
    """Operator shape of the reference's GPT2Wrapper (src/gpt/lower_gpt_model.py:20-50): full logits
    [B, S, V] for (input_ids, attention_mask), here backed by the B200 library."""

    def __init__(self, cfg: Gpt2Config | None = None, seed: int = 1234, init_mode: int = 0,
                 blob: np.ndarray | None = None, device: int = -1):
        self.cfg = cfg or gpt2_small()
        init(self.cfg, device)
        if blob is not None:
            load_weights(blob)
        else:
            init_seeded(seed, init_mode)

    def forward(self, input_ids, attention_mask=None) -> np.ndarray:
        return forward_host(input_ids, attention_mask)

    __call__ = forward


# ---------------------------------------------------------------------------
# kernel-level entry points (device pointers as ints)
# ---------------------------------------------------------------------------
def k_gemm_f32(A, B, b_nk, C, M, N, K, ldc, bias=None, resid=None, epi=EPI_NONE, stream=None):
    _check(lib().gpt2k_gemm_f32(A, B, b_nk, C, M, N, K, ldc, bias, resid, epi, stream), "gpt2k_gemm_f32")


def k_gemm_bf16(A, B, C, M, N, K, ldc, out_f32=0, bias=None, resid=None, epi=EPI_NONE, bn=256, stream=None):
    _check(lib().gpt2k_gemm_bf16(A, B, C, M, N, K, ldc, out_f32, bias, resid, epi, bn, stream), "gpt2k_gemm_bf16")


def k_gemv_bf16(x, W, y, M, N, K, ldy, bias=None, resid=None, epi=EPI_NONE, ln_gain=None, ln_shift=None,
                eps=1e-5, out_f32=0, impl=1, stream=None):
    """gpt2k_gemv_bf16: y = epi(LN(x) @ W^T) for M <= 16 rows; impl 0 SIMT, 1 tensor cores (device pointers)."""
    _check(lib().gpt2k_gemv_bf16(x, W, y, M, N, K, ldy, bias, resid, epi, ln_gain, ln_shift, eps, out_f32, impl,
                                 stream), "gpt2k_gemv_bf16")


def k_test_gemm_withheld_load(A, B, C, M, N, K, status_ptr, stream=None):
    """gpt2k_test_gemm_withheld_load: the tcgen05 GEMM with one TMA copy withheld (timeout-path test hook)."""
    _check(lib().gpt2k_test_gemm_withheld_load(A, B, C, M, N, K, status_ptr, stream), "gpt2k_test_gemm_withheld_load")


def k_gemm_bf16_ln(A, B, C, M, N, K, ldc, out_f32=0, bias=None, resid=None, epi=EPI_LN_BIAS, bn=256, c1=None,
                   c2=None, stats_in=None, stats_out=None, eps=1e-5, stream=None):
    _check(lib().gpt2k_gemm_bf16_ln(A, B, C, M, N, K, ldc, out_f32, bias, resid, epi, bn, c1, c2, stats_in,
                                    stats_out, eps, stream), "gpt2k_gemm_bf16_ln")


def k_ln_fold_pack(W, w_kn, gain, shift, bias, B, c1, c2, N, K, stream=None):
    _check(lib().gpt2k_ln_fold_pack(W, w_kn, gain, shift, bias, B, c1, c2, N, K, stream), "gpt2k_ln_fold_pack")


def k_ffma_peak(stream=None) -> float:
    """Measured FP32 FFMA throughput of the current device, TFLOP/s."""
    v = ctypes.c_float(0.0)
    _check(lib().gpt2k_ffma_peak(ctypes.byref(v), stream), "gpt2k_ffma_peak")
    return float(v.value)


def k_layernorm(x, gain, shift, y, T, d, eps, dtype, stream=None):
    _check(lib().gpt2k_layernorm(x, gain, shift, y, T, d, eps, dtype, stream), "gpt2k_layernorm")


def k_attention_workspace_bytes(B, S) -> int:
    return int(lib().gpt2k_attention_workspace_bytes(B, S))


def k_attention(qkv, mask, o, B, S, H, dtype, workspace=None, stream=None):
    _check(lib().gpt2k_attention(qkv, mask, o, B, S, H, dtype, workspace, stream), "gpt2k_attention")


def k_attention_ex_workspace_bytes(B, S) -> int:
    return int(lib().gpt2k_attention_ex_workspace_bytes(B, S))


def k_attention_ex(qkv, mask, o, B, S, H, dtype, causal, workspace=None, stream=None):
    _check(lib().gpt2k_attention_ex(qkv, mask, o, B, S, H, dtype, causal, workspace, stream), "gpt2k_attention_ex")


def k_attention_noalloc(qkv, mask, o, B, S, H, dtype, stream=None):
    _check(lib().gpt2k_attention_noalloc(qkv, mask, o, B, S, H, dtype, stream), "gpt2k_attention_noalloc")


def k_embed(ids, wte, wpe, x, T, S, d, V, dtype, status_ptr=None, stream=None):
    _check(lib().gpt2k_embed(ids, wte, wpe, x, T, S, d, V, dtype, status_ptr, stream), "gpt2k_embed")


from . import bert  # noqa: E402  (the BERT encoder entry points, include/bert_b200.h)
