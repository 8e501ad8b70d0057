"""Python host mirror of the BERT entry points of libgpt2_b200.so
(include/bert_b200.h).

The reference exports transformers' BertModel wrapped as
Wrapper.forward(input_ids, token_type_ids, attention_mask) ->
(last_hidden_state, pooler_output) (src/bert-base-uncased/lower_bert_model.py:7-18)
and calls it through `_mlir_ciface_bert_model` with the model's position-id
and token-type buffers prepended (src/bert-base-uncased/call_bert.cpp:41-53,
:73-116).  This module binds:

  * `bert_model(ids, token_type_ids, mask, position_ids=..., token_type_buffer=...)`:
    the drop-in symbol, numpy int64 [B, S] in, (hidden [B, S, d], pooled [B, d]) out;
  * `BertModel(...).forward(input_ids, token_type_ids, attention_mask)`: the
    wrapper's operator shape;
  * `forward_device` / `forward_host` for device pointers and host buffers.

No CPU fallback: every call goes to the CUDA library.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import DTYPE_BF16, DTYPE_F32, Gpt2Error, MemRef2D_i64, MemRef3D, _libc, lib as _lib

KERNEL_KINDS = ["seq_info", "embed_ln", "layernorm", "gemm_qkv", "attention", "masked_rows", "gemm_attn_out",
                "gemm_intermediate", "gemm_output", "pooler"]


class BertConfig(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int32),
        ("n_embd", ctypes.c_int32),
        ("n_head", ctypes.c_int32),
        ("n_inner", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("n_positions", ctypes.c_int32),
        ("layer_norm_eps", ctypes.c_float),
        ("type_vocab", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class MemRef2D_f32(ctypes.Structure):
    _fields_ = [
        ("allocated", ctypes.POINTER(ctypes.c_float)),
        ("aligned", ctypes.POINTER(ctypes.c_float)),
        ("offset", ctypes.c_int64),
        ("sizes", ctypes.c_int64 * 2),
        ("strides", ctypes.c_int64 * 2),
    ]


class BertOutput(ctypes.Structure):
    _fields_ = [("last_hidden_state", MemRef3D), ("pooler_output", MemRef2D_f32)]


def bert_base(dtype: int = DTYPE_F32) -> BertConfig:
    """bert-base-uncased: 12 layers, d 768, 12 heads of 64, intermediate 3072, vocab 30522, 512 positions."""
    return BertConfig(12, 768, 12, 3072, 30522, 512, 1e-12, 2, dtype)


_bound = False


def lib() -> ctypes.CDLL:
    global _bound
    L = _lib()
    if _bound:
        return L
    P, i64, i32, vp = ctypes.POINTER, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    L._mlir_ciface_bert_model.restype = None
    L._mlir_ciface_bert_model.argtypes = [P(BertOutput)] + [P(MemRef2D_i64)] * 5
    L.bert_init.argtypes = [P(BertConfig), i32]
    L.bert_blob_floats.argtypes = [P(BertConfig)]
    L.bert_blob_floats.restype = i64
    L.bert_load_weights.argtypes = [vp, ctypes.c_size_t, ctypes.c_char_p]
    L.bert_init_seeded.argtypes = [ctypes.c_uint64, i32]
    L.bert_seeded_blob.argtypes = [P(BertConfig), ctypes.c_uint64, i32, P(ctypes.c_float)]
    L.bert_get_config.argtypes = [P(BertConfig)]
    L.bert_shutdown.restype = None
    L.bert_last_error.restype = ctypes.c_char_p
    L.bert_safetensors_to_blob.argtypes = [ctypes.c_char_p, P(BertConfig), P(ctypes.c_float)]
    L.bert_load_safetensors.argtypes = [ctypes.c_char_p]
    L.bert_forward_device.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp, vp]
    L.bert_forward_host.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp]
    L.bert_forward_launches.argtypes = [i32, i32]
    L.bert_profile_end.argtypes = [P(ctypes.c_double), P(i64), i32]
    _bound = True
    return L


def last_error() -> str:
    return lib().bert_last_error().decode()


def _check(rc: int, what: str) -> int:
    if rc < 0:
        raise Gpt2Error(f"{what} failed ({rc}): {last_error()}")
    return rc


def init(cfg: BertConfig, device: int = -1) -> None:
    _check(lib().bert_init(ctypes.byref(cfg), device), "bert_init")


def get_config() -> BertConfig:
    cfg = BertConfig()
    _check(lib().bert_get_config(ctypes.byref(cfg)), "bert_get_config")
    return cfg


def blob_floats(cfg: BertConfig) -> int:
    return _check(lib().bert_blob_floats(ctypes.byref(cfg)), "bert_blob_floats")


def seeded_blob(cfg: BertConfig, seed: int, init_mode: int = 0) -> np.ndarray:
    out = np.empty(blob_floats(cfg), dtype=np.float32)
    _check(lib().bert_seeded_blob(ctypes.byref(cfg), seed, init_mode,
                                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "bert_seeded_blob")
    return out


def load_weights(blob: np.ndarray, manifest: str | None = None) -> None:
    blob = np.ascontiguousarray(blob, dtype=np.float32)
    _check(lib().bert_load_weights(blob.ctypes.data, blob.nbytes, manifest.encode() if manifest else None),
           "bert_load_weights")


def safetensors_to_blob(path: str, cfg: BertConfig) -> np.ndarray:
    """The canonical FP32 blob of an HF BERT safetensors checkpoint (no GPU needed)."""
    out = np.empty(blob_floats(cfg), dtype=np.float32)
    _check(lib().bert_safetensors_to_blob(os.fsencode(path), ctypes.byref(cfg),
                                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))), "bert_safetensors_to_blob")
    return out


def load_safetensors(path: str) -> None:
    _check(lib().bert_load_safetensors(os.fsencode(path)), "bert_load_safetensors")


def init_seeded(seed: int, init_mode: int = 0) -> None:
    _check(lib().bert_init_seeded(seed, init_mode), "bert_init_seeded")


def shutdown() -> None:
    lib().bert_shutdown()


def status() -> int:
    return lib().bert_status()


def forward_launches(has_mask: bool, has_pooler: bool = True) -> int:
    return _check(lib().bert_forward_launches(int(has_mask), int(has_pooler)), "bert_forward_launches")


def _i64(a) -> np.ndarray:
    a = np.asarray(a, dtype=np.int64)
    if a.ndim != 2:
        raise ValueError("BERT inputs are [B, S]")
    return a


def _desc(a: np.ndarray) -> MemRef2D_i64:
    p = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
    return MemRef2D_i64(p, p, 0, (ctypes.c_int64 * 2)(*a.shape),
                        (ctypes.c_int64 * 2)(a.strides[0] // a.itemsize, a.strides[1] // a.itemsize))


def bert_model(input_ids, token_type_ids=None, attention_mask=None, position_ids=None, token_type_buffer=None):
    """Calls `_mlir_ciface_bert_model` as src/bert-base-uncased/call_bert.cpp:110-116 does: the
    position-id and token-type buffers ([1, n_positions], default arange / zeros as transformers
    registers them), then ids, token types and mask; strides honoured; the malloc'd results are
    copied out and freed.  token_type_ids None passes a null descriptor (the buffer applies)."""
    ids = _i64(input_ids)
    n = max(512, ids.shape[1])
    pos = _i64(position_ids) if position_ids is not None else np.arange(n, dtype=np.int64)[None]
    ttb = _i64(token_type_buffer) if token_type_buffer is not None else np.zeros((1, n), dtype=np.int64)
    mask = _i64(attention_mask) if attention_mask is not None else np.ones_like(ids)
    keep = [ids, pos, ttb, mask]
    d_pos, d_ttb, d_ids, d_mask = _desc(pos), _desc(ttb), _desc(ids), _desc(mask)
    d_tt = None
    if token_type_ids is not None:
        tt = _i64(token_type_ids)
        keep.append(tt)
        d_tt = _desc(tt)
    res = BertOutput()
    lib()._mlir_ciface_bert_model(ctypes.byref(res), ctypes.byref(d_pos), ctypes.byref(d_ttb), ctypes.byref(d_ids),
                                  ctypes.byref(d_tt) if d_tt is not None else None, ctypes.byref(d_mask))
    del keep
    h, p = res.last_hidden_state, res.pooler_output
    if not h.allocated or not p.allocated:
        raise Gpt2Error(f"_mlir_ciface_bert_model failed: {last_error()}")
    hs = tuple(h.sizes)
    hidden = np.ctypeslib.as_array(h.aligned, shape=(hs[0] * hs[1] * hs[2],)).reshape(hs).copy()
    pooled = np.ctypeslib.as_array(p.aligned, shape=(p.sizes[0] * p.sizes[1],)).reshape(p.sizes[0], p.sizes[1]).copy()
    _libc.free(ctypes.cast(h.allocated, ctypes.c_void_p))
    _libc.free(ctypes.cast(p.allocated, ctypes.c_void_p))
    return hidden, pooled


def forward_host(input_ids, token_type_ids=None, attention_mask=None, position_ids=None, pooler: bool = True):
    ids = np.ascontiguousarray(_i64(input_ids))
    B, S = ids.shape
    d = get_config().n_embd
    arrs = {}
    for k, a in (("tt", token_type_ids), ("mask", attention_mask)):
        arrs[k] = None if a is None else np.ascontiguousarray(_i64(a))
    pos = None if position_ids is None else np.ascontiguousarray(np.asarray(position_ids, dtype=np.int64).ravel()[:S])
    hidden = np.empty((B, S, d), dtype=np.float32)
    pooled = np.empty((B, d), dtype=np.float32) if pooler else None
    ptr = lambda a: None if a is None else a.ctypes.data  # noqa: E731
    _check(lib().bert_forward_host(ptr(ids), ptr(arrs["tt"]), ptr(pos), ptr(arrs["mask"]), B, S, ptr(hidden),
                                   ptr(pooled)), "bert_forward_host")
    return hidden, pooled


def forward_device(ids_ptr, tt_ptr, pos_ptr, mask_ptr, B: int, S: int, hidden_ptr, pooled_ptr, stream_ptr=None):
    _check(lib().bert_forward_device(ids_ptr, tt_ptr, pos_ptr, mask_ptr, B, S, hidden_ptr, pooled_ptr, stream_ptr),
           "bert_forward_device")


def profile_begin() -> None:
    _check(lib().bert_profile_begin(), "bert_profile_begin")


def profile_end() -> dict:
    n = len(KERNEL_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int64 * n)()
    _check(lib().bert_profile_end(ms, cnt, n), "bert_profile_end")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(KERNEL_KINDS)}


class BertModel:
    """Operator shape of the reference's export wrapper (src/bert-base-uncased/lower_bert_model.py:7-18):
    (last_hidden_state, pooler_output) for (input_ids, token_type_ids, attention_mask)."""

    def __init__(self, cfg: BertConfig | None = None, seed: int = 1234, init_mode: int = 0,
                 blob: np.ndarray | None = None, device: int = -1):
        self.cfg = cfg or bert_base()
        init(self.cfg, device)
        if blob is not None:
            load_weights(blob)
        else:
            init_seeded(seed, init_mode)

    def forward(self, input_ids, token_type_ids=None, attention_mask=None):
        return forward_host(input_ids, token_type_ids, attention_mask)

    __call__ = forward


__all__ = ["BertConfig", "BertModel", "BertOutput", "MemRef2D_f32", "bert_base", "bert_model", "forward_host",
           "forward_device", "init", "load_weights", "init_seeded", "seeded_blob", "shutdown", "status",
           "DTYPE_F32", "DTYPE_BF16"]
