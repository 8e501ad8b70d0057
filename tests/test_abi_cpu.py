"""CPU tests of the C ABI library: it loads without a GPU, exports every
function include/gpt2_b200.h and include/bert_b200.h declare, its host-side
seeded generators match
the oracle's bit for bit, and without a GPU every entry point fails with an
error code instead of aborting."""
import ctypes
import subprocess

import numpy as np
import pytest

from helpers import load_oracle, load_pkg, shape_to_cfg

pkg = load_pkg()
O = load_oracle()


def test_library_exports_every_declared_function():
    lib = pkg.lib()
    declared = pkg.declared_functions()
    assert "gpt2_decoder" in declared and "_mlir_ciface_gpt2_decoder" in declared
    assert "_mlir_ciface_bert_model" in declared
    missing = [f for f in declared if not hasattr(lib, f)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(declared) <= exported
    # only the C ABI is exported (static cudart and C++ internals stay hidden)
    assert all(s.startswith(("gpt2_", "gpt2k_", "bert_", "_mlir_ciface_gpt2", "_mlir_ciface_bert")) for s in exported), \
        exported


def test_memref_struct_layout():
    # 72-byte result struct of src/gpt/gpt2_call.cpp:23-29 (two pointers, offset, sizes[3], strides[3])
    assert ctypes.sizeof(pkg.MemRef3D) == 72
    assert ctypes.sizeof(pkg.MemRef2D_i64) == 56
    assert ctypes.sizeof(pkg.Gpt2Config) == 32
    # result struct of src/bert-base-uncased/call_bert.cpp:41-44: a 3-D and a 2-D f32 memref
    assert ctypes.sizeof(pkg.bert.MemRef2D_f32) == 56
    assert ctypes.sizeof(pkg.bert.BertOutput) == 72 + 56
    assert ctypes.sizeof(pkg.bert.BertConfig) == 36


@pytest.mark.parametrize("shape_name,mode", [("BERT_TINY", 0), ("BERT_TINY", 1), ("BERT_BASE", 1)])
def test_bert_seeded_blob_matches_oracle(shape_name, mode):
    shape = getattr(O, shape_name)
    cfg = pkg.bert.BertConfig(shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                              shape.n_positions, shape.layer_norm_eps, shape.type_vocab, 0)
    assert pkg.bert.blob_floats(cfg) == int(O.bert_blob_layout(shape)[-1])
    a = pkg.bert.seeded_blob(cfg, 77, mode)
    b = O.bert_seeded_blob(shape, 77, mode)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("shape_name,mode", [("GPT2_TINY", 0), ("GPT2_TINY", 1), ("GPT2_SMALL", 0)])
def test_seeded_blob_matches_oracle(shape_name, mode):
    shape = getattr(O, shape_name)
    cfg = shape_to_cfg(pkg, shape, pkg.DTYPE_F32)
    assert pkg.blob_floats(cfg) == int(O.blob_layout(shape)[-1])
    a = pkg.seeded_blob(cfg, 1234, mode)
    b = O.seeded_blob(shape, 1234, mode)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_seeded_ids_match_oracle():
    a = pkg.seeded_ids(2, 333, 99, 50257)
    b = O.token_ids(2, 333, 99, 50257)
    assert np.array_equal(a, b)


def _no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU error paths")
def test_entry_points_fail_cleanly_without_gpu():
    lib = pkg.lib()
    cfg = pkg.gpt2_small()
    rc = lib.gpt2_init(ctypes.byref(cfg), -1)
    assert rc < 0 and pkg.last_error()
    with pytest.raises(pkg.Gpt2Error):
        pkg.gpt2_decoder(np.array([[464, 3139, 286, 4881, 318]]))
    with pytest.raises(pkg.Gpt2Error):
        pkg.ciface_gpt2_decoder(np.array([[464, 3139]]))
    assert pkg.status() < 0
    assert lib.gpt2_forward_device(None, None, 1, 5, None, 50257, 0, None) < 0
    # the BERT entry points: error code / zeroed result, no abort
    B = pkg.bert
    assert B.lib().bert_init(ctypes.byref(B.bert_base()), -1) < 0 and B.last_error()
    with pytest.raises(pkg.Gpt2Error):
        B.bert_model(np.array([[101, 2023, 102]]))
    assert B.status() < 0
    assert B.lib().bert_forward_device(None, None, None, None, 1, 3, None, None, None) < 0


def test_argument_validation_needs_no_gpu():
    lib = pkg.lib()
    bad = pkg.Gpt2Config(0, 768, 12, 3072, 50257, 1024, 1e-5, 0)
    assert lib.gpt2_init(ctypes.byref(bad), -1) == -1
    assert lib.gpt2_blob_floats(ctypes.byref(bad)) == -1
    assert lib.gpt2_seeded_ids(None, 4, 1, 0, 10) == -1
    bad_bert = pkg.bert.BertConfig(12, 768, 12, 3072, 30522, 512, 1e-12, 0, 0)  # no token types
    assert pkg.bert.lib().bert_init(ctypes.byref(bad_bert), -1) == -1
    assert pkg.bert.lib().bert_blob_floats(ctypes.byref(bad_bert)) == -1
