"""ctypes wrapper around the CPU oracle (oracle/gpt2_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, the smoke() entry and bench.py's
cpu_baseline / reference legs import this module to check or time the
product; the product path never does.

The oracle restates the reference's GPT-2 forward (HF GPT-2 as wrapped by
src/gpt/lower_gpt_model.py:20-50 and lowered for the CPU by
src/gpt/run_mlir_pipeline.sh:5-10, matmuls through cblas_sgemm as
lib/ConvertMatMulToBlas.cpp:156-160 emits them).  It is pinned against
transformers' GPT2LMHeadModel by the fixtures in tests/golden/.
"""
from __future__ import annotations

import ctypes
import glob
import os
import subprocess
import sys
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libgpt2_oracle.so")

# Philox stream used for the seeded token ids (weights use streams 0..4+12L).
IDS_STREAM = 0x10000


class OracleCfg(ctypes.Structure):
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


@dataclass(frozen=True)
class ModelShape:
    n_layer: int = 12
    n_embd: int = 768
    n_head: int = 12
    n_inner: int = 3072
    vocab_size: int = 50257
    n_positions: int = 1024
    layer_norm_eps: float = 1e-5

    def c(self) -> OracleCfg:
        return OracleCfg(self.n_layer, self.n_embd, self.n_head, self.n_inner,
                         self.vocab_size, self.n_positions, self.layer_norm_eps, 0)


class OracleBertCfg(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int32),
        ("n_embd", ctypes.c_int32),
        ("n_head", ctypes.c_int32),
        ("n_inner", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("n_positions", ctypes.c_int32),
        ("layer_norm_eps", ctypes.c_float),
        ("type_vocab", ctypes.c_int32),
    ]


@dataclass(frozen=True)
class BertShape:
    n_layer: int = 12
    n_embd: int = 768
    n_head: int = 12
    n_inner: int = 3072
    vocab_size: int = 30522
    n_positions: int = 512
    layer_norm_eps: float = 1e-12
    type_vocab: int = 2

    def c(self) -> OracleBertCfg:
        return OracleBertCfg(self.n_layer, self.n_embd, self.n_head, self.n_inner, self.vocab_size,
                             self.n_positions, self.layer_norm_eps, self.type_vocab)


BERT_BASE = BertShape()
BERT_TINY = BertShape(n_layer=2, n_embd=128, n_head=2, n_inner=512, vocab_size=1000, n_positions=64)
GPT2_SMALL = ModelShape()
# A small model of the same family for fast, mask-heavy parity cases.
GPT2_TINY = ModelShape(n_layer=2, n_embd=128, n_head=2, n_inner=512, vocab_size=1000, n_positions=64)

_lib = None


def build(quiet: bool = True) -> str:
    """Compiles the oracle with its Makefile; returns the library path."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        sys.stdout.write(out.stdout)
    return LIB_PATH


def find_openblas() -> str | None:
    """The OpenBLAS that scipy bundles (LP64 `scipy_cblas_sgemm`), else numpy's (ILP64)."""
    try:
        import scipy  # noqa: F401
        base = os.path.dirname(os.path.dirname(scipy.__file__))
        hits = sorted(glob.glob(os.path.join(base, "scipy.libs", "libscipy_openblas-*.so")))
        if hits:
            return hits[0]
    except ImportError:
        pass
    base = os.path.dirname(os.path.dirname(np.__file__))
    hits = sorted(glob.glob(os.path.join(base, "numpy.libs", "libscipy_openblas64_*.so")))
    return hits[0] if hits else None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    L.oracle_num_tensors.argtypes = [P(OracleCfg)]
    L.oracle_num_tensors.restype = ctypes.c_int
    L.oracle_blob_layout.argtypes = [P(OracleCfg), P(ctypes.c_int64)]
    L.oracle_blob_layout.restype = ctypes.c_int64
    L.oracle_philox4x32_10.argtypes = [P(ctypes.c_uint32), P(ctypes.c_uint32), P(ctypes.c_uint32)]
    L.oracle_normal_fill.argtypes = [P(ctypes.c_float), ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
                                     ctypes.c_double, ctypes.c_double]
    L.oracle_token_ids.argtypes = [P(ctypes.c_int64), ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
                                   ctypes.c_int64]
    L.oracle_seeded_blob.argtypes = [P(OracleCfg), ctypes.c_uint64, ctypes.c_int, P(ctypes.c_float)]
    L.oracle_seeded_blob.restype = ctypes.c_int
    L.oracle_set_blas.argtypes = [ctypes.c_char_p]
    L.oracle_set_blas.restype = ctypes.c_int
    L.oracle_blas_name.restype = ctypes.c_char_p
    L.oracle_set_loop_threads.argtypes = [ctypes.c_int]
    L.oracle_gpt2_forward.argtypes = [P(OracleCfg), P(ctypes.c_float), P(ctypes.c_int64), P(ctypes.c_int64),
                                      ctypes.c_int, ctypes.c_int, P(ctypes.c_float)]
    L.oracle_gpt2_forward.restype = ctypes.c_int
    L.oracle_e4m3_encode.argtypes = [ctypes.c_float]
    L.oracle_e4m3_encode.restype = ctypes.c_uint8
    L.oracle_e4m3_decode.argtypes = [ctypes.c_uint8]
    L.oracle_e4m3_decode.restype = ctypes.c_float
    L.oracle_fp8_quantize.argtypes = [P(ctypes.c_float), ctypes.c_int, ctypes.c_int, P(ctypes.c_uint8), P(ctypes.c_float)]
    L.oracle_fp8_dequantize_blob.argtypes = [P(OracleCfg), P(ctypes.c_float)]
    L.oracle_fp8_dequantize_blob.restype = ctypes.c_int
    L.oracle_bert_num_tensors.argtypes = [P(OracleBertCfg)]
    L.oracle_bert_blob_layout.argtypes = [P(OracleBertCfg), P(ctypes.c_int64)]
    L.oracle_bert_blob_layout.restype = ctypes.c_int64
    L.oracle_bert_seeded_blob.argtypes = [P(OracleBertCfg), ctypes.c_uint64, ctypes.c_int, P(ctypes.c_float)]
    L.oracle_bert_forward.argtypes = [P(OracleBertCfg), P(ctypes.c_float), P(ctypes.c_int64), P(ctypes.c_int64),
                                      P(ctypes.c_int64), P(ctypes.c_int64), ctypes.c_int, ctypes.c_int,
                                      P(ctypes.c_float), P(ctypes.c_float)]
    L.oracle_bert_forward.restype = ctypes.c_int
    blas = os.environ.get("ORACLE_BLAS", None)
    if blas is None:
        blas = find_openblas() or ""
    if blas and L.oracle_set_blas(blas.encode()) != 0:
        L.oracle_set_blas(b"")
    _lib = L
    return L


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def blas_name() -> str:
    return lib().oracle_blas_name().decode()


def set_loop_threads(n: int) -> None:
    lib().oracle_set_loop_threads(int(n))


def philox(ctr, key) -> np.ndarray:
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(_ptr(c, ctypes.c_uint32), _ptr(k, ctypes.c_uint32), _ptr(out, ctypes.c_uint32))
    return out


def normal_fill(n: int, seed: int, stream: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_normal_fill(_ptr(out, ctypes.c_float), n, seed, stream, mean, std)
    return out


def token_ids(B: int, S: int, seed: int, vocab: int, stream: int = IDS_STREAM) -> np.ndarray:
    out = np.empty(B * S, dtype=np.int64)
    lib().oracle_token_ids(_ptr(out, ctypes.c_int64), B * S, seed, stream, vocab)
    return out.reshape(B, S)


def blob_layout(shape: ModelShape) -> np.ndarray:
    c = shape.c()
    n = lib().oracle_num_tensors(ctypes.byref(c))
    off = np.zeros(n + 1, dtype=np.int64)
    lib().oracle_blob_layout(ctypes.byref(c), _ptr(off, ctypes.c_int64))
    return off


def seeded_blob(shape: ModelShape, seed: int, init_mode: int = 0) -> np.ndarray:
    c = shape.c()
    total = int(lib().oracle_blob_layout(ctypes.byref(c), None))
    blob = np.empty(total, dtype=np.float32)
    rc = lib().oracle_seeded_blob(ctypes.byref(c), seed, init_mode, _ptr(blob, ctypes.c_float))
    assert rc == 0
    return blob


def tensor_names(shape: ModelShape) -> list[str]:
    names = ["transformer.wte.weight", "transformer.wpe.weight"]
    per = ["ln_1.weight", "ln_1.bias", "attn.c_attn.weight", "attn.c_attn.bias", "attn.c_proj.weight",
           "attn.c_proj.bias", "ln_2.weight", "ln_2.bias", "mlp.c_fc.weight", "mlp.c_fc.bias",
           "mlp.c_proj.weight", "mlp.c_proj.bias"]
    for l in range(shape.n_layer):
        names += [f"transformer.h.{l}.{p}" for p in per]
    names += ["transformer.ln_f.weight", "transformer.ln_f.bias"]
    return names


# GPT-2 XL-shaped model of the weight-only FP8 configuration.
GPT2_XL = ModelShape(n_layer=48, n_embd=1600, n_head=25, n_inner=6400)


def fp8_quantize(w: np.ndarray):
    """Conv1D weight w [K, N] -> (q [N, K] uint8 E4M3 codes, scale [N])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    K, N = w.shape
    q = np.empty((N, K), dtype=np.uint8)
    sc = np.empty(N, dtype=np.float32)
    lib().oracle_fp8_quantize(_ptr(w, ctypes.c_float), K, N, _ptr(q, ctypes.c_uint8), _ptr(sc, ctypes.c_float))
    return q, sc


def fp8_dequantized_blob(shape: ModelShape, blob: np.ndarray) -> np.ndarray:
    """Copy of the blob whose Conv1D weights are replaced by their FP8-dequantized values."""
    out = np.array(blob, dtype=np.float32, copy=True)
    c = shape.c()
    assert lib().oracle_fp8_dequantize_blob(ctypes.byref(c), _ptr(out, ctypes.c_float)) == 0
    return out


def forward(shape: ModelShape, blob: np.ndarray, ids: np.ndarray, mask: np.ndarray | None = None,
            out: np.ndarray | None = None) -> np.ndarray:
    """FP32 logits [B, S, V] of the GPT-2 forward on (ids, mask)."""
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    B, S = ids.shape
    if out is None:
        out = np.empty((B, S, shape.vocab_size), dtype=np.float32)
    m = None
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.int64)
        m = _ptr(mask, ctypes.c_int64)
    c = shape.c()
    rc = lib().oracle_gpt2_forward(ctypes.byref(c), _ptr(blob, ctypes.c_float), _ptr(ids, ctypes.c_int64), m,
                                   B, S, _ptr(out, ctypes.c_float))
    if rc != 0:
        raise ValueError(f"oracle_gpt2_forward failed with code {rc}")
    return out


def _top(x: np.ndarray, k: int) -> np.ndarray:
    """Column indices of each row's k largest entries, largest first (ties: lower index first)."""
    part = np.argpartition(-x, k - 1, axis=1)[:, :k]
    vals = np.take_along_axis(x, part, axis=1)
    order = np.lexsort((part, -vals), axis=1)
    return np.take_along_axis(part, order, axis=1)


def top5_report(ref: np.ndarray, got: np.ndarray, bound: float) -> dict:
    """Top-5 agreement of logits `got` with the oracle's `ref` (both [..., V]) under a STATED
    per-logit error bound (an absolute logit difference fixed by the caller, not measured on
    these rows).

    A position is checkable when each of the oracle's top five logits leads the next one (1st
    over 2nd, ..., 5th over 6th) by more than 2 * bound: two logits that are each within
    `bound` of the oracle cannot swap there, so a kernel that honours the bound must give the
    same five ids in the same order.  Reported:
      total, checked (checkable positions), identical (checkable positions whose top-5 ids and
      order agree), top1 (fraction of ALL positions whose argmax agrees), overlap (mean size of
      the intersection of the two top-5 sets over ALL positions, 0..5), exceed (fraction of all
      logits farther than `bound` from the oracle), max_err, p999 (99.9th percentile of the
      per-logit error) and the bound itself."""
    V = ref.shape[-1]
    r = np.ascontiguousarray(ref, dtype=np.float32).reshape(-1, V)
    g = np.ascontiguousarray(got, dtype=np.float32).reshape(-1, V)
    ri = _top(r, 6)
    rv = np.take_along_axis(r, ri, axis=1)
    checkable = (rv[:, :5] - rv[:, 1:6] > 2.0 * bound).all(axis=1)
    gi = _top(g, 5)
    same = (gi == ri[:, :5]).all(axis=1)
    err = np.abs(g - r)
    return {
        "total": int(r.shape[0]),
        "checked": int(checkable.sum()),
        "identical": int((same & checkable).sum()),
        "top1": float((gi[:, 0] == ri[:, 0]).mean()),
        "overlap": float((gi[:, :, None] == ri[:, None, :5]).any(axis=2).sum(axis=1).mean()),
        "exceed": float((err > bound).mean()),
        "max_err": float(err.max()),
        "p999": float(np.quantile(err, 0.999)),
        "bound": float(bound),
    }


# ---------------------------------------------------------------------------
# BERT encoder
# ---------------------------------------------------------------------------
BERT_IDS_STREAM = 0x30000


def bert_blob_layout(shape: BertShape) -> np.ndarray:
    c = shape.c()
    n = lib().oracle_bert_num_tensors(ctypes.byref(c))
    off = np.zeros(n + 1, dtype=np.int64)
    lib().oracle_bert_blob_layout(ctypes.byref(c), _ptr(off, ctypes.c_int64))
    return off


def bert_seeded_blob(shape: BertShape, seed: int, init_mode: int = 0) -> np.ndarray:
    c = shape.c()
    total = int(lib().oracle_bert_blob_layout(ctypes.byref(c), None))
    blob = np.empty(total, dtype=np.float32)
    lib().oracle_bert_seeded_blob(ctypes.byref(c), seed, init_mode, _ptr(blob, ctypes.c_float))
    return blob


def bert_tensor_names(shape: BertShape) -> list[str]:
    names = ["embeddings.word_embeddings.weight", "embeddings.position_embeddings.weight",
             "embeddings.token_type_embeddings.weight", "embeddings.LayerNorm.weight", "embeddings.LayerNorm.bias"]
    per = ["attention.self.query.weight", "attention.self.query.bias", "attention.self.key.weight",
           "attention.self.key.bias", "attention.self.value.weight", "attention.self.value.bias",
           "attention.output.dense.weight", "attention.output.dense.bias", "attention.output.LayerNorm.weight",
           "attention.output.LayerNorm.bias", "intermediate.dense.weight", "intermediate.dense.bias",
           "output.dense.weight", "output.dense.bias", "output.LayerNorm.weight", "output.LayerNorm.bias"]
    for l in range(shape.n_layer):
        names += [f"encoder.layer.{l}.{p}" for p in per]
    names += ["pooler.dense.weight", "pooler.dense.bias"]
    return names


def bert_forward(shape: BertShape, blob: np.ndarray, ids: np.ndarray, token_type_ids: np.ndarray | None = None,
                 mask: np.ndarray | None = None, position_ids: np.ndarray | None = None):
    """(last_hidden_state [B, S, d], pooler_output [B, d]) in FP32."""
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    B, S = ids.shape
    hidden = np.empty((B, S, shape.n_embd), dtype=np.float32)
    pooled = np.empty((B, shape.n_embd), dtype=np.float32)
    args = []
    for a in (token_type_ids, position_ids, mask):
        if a is None:
            args.append(None)
        else:
            a = np.ascontiguousarray(a, dtype=np.int64)
            args.append(a)
    ptrs = [None if a is None else _ptr(a, ctypes.c_int64) for a in args]
    c = shape.c()
    rc = lib().oracle_bert_forward(ctypes.byref(c), _ptr(blob, ctypes.c_float), _ptr(ids, ctypes.c_int64), ptrs[0],
                                   ptrs[1], ptrs[2], B, S, _ptr(hidden, ctypes.c_float), _ptr(pooled, ctypes.c_float))
    if rc != 0:
        raise ValueError(f"oracle_bert_forward failed with code {rc}")
    return hidden, pooled
