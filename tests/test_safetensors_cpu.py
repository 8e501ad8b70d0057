"""CPU tests of the safetensors ingestion (gpt2_safetensors_to_blob,
bert_safetensors_to_blob): checkpoints written by transformers'
save_pretrained and by the safetensors package, in F32, F16 and BF16, with
and without the model prefix, map onto the canonical blob exactly."""
import os

import numpy as np
import pytest

from helpers import load_oracle, load_pkg, shape_to_cfg

pkg = load_pkg()
O = load_oracle()
torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")
st_torch = pytest.importorskip("safetensors.torch")


def _gpt2_hf(shape, blob):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_golden import hf_model
    return hf_model(shape, blob)


def _bert_hf(shape, blob):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_golden import hf_bert
    return hf_bert(shape, blob)


def _bert_cfg(shape):
    return pkg.bert.BertConfig(shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                               shape.n_positions, shape.layer_norm_eps, shape.type_vocab, 0)


def test_gpt2_save_pretrained_roundtrip(tmp_path):
    """GPT2LMHeadModel.save_pretrained (names with "transformer.", tied lm_head dropped, attn.bias
    buffers absent or ignored) reads back bit for bit."""
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 31, 1)
    model = _gpt2_hf(shape, blob)
    model.save_pretrained(tmp_path, safe_serialization=True)
    got = pkg.safetensors_to_blob(str(tmp_path / "model.safetensors"), shape_to_cfg(pkg, shape, 0))
    assert np.array_equal(got.view(np.uint32), blob.view(np.uint32))


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_gpt2_hub_layout_and_16_bit_dtypes(tmp_path, dtype):
    """The hub gpt2 layout (names without a prefix, plus the h.N.attn.bias mask buffers) in F32,
    F16 and BF16: 16-bit values widen exactly."""
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 32, 1)
    sd = _gpt2_hf(shape, blob).state_dict()
    td = getattr(torch, dtype)
    out = {}
    for k, v in sd.items():
        if k == "lm_head.weight":
            continue
        out[k.removeprefix("transformer.")] = v.to(td).contiguous() if v.is_floating_point() else v.contiguous()
    for l in range(shape.n_layer):
        out[f"h.{l}.attn.bias"] = torch.ones(1, 1, shape.n_positions, shape.n_positions, dtype=td)
    path = str(tmp_path / "gpt2.safetensors")
    st_torch.save_file(out, path, metadata={"format": "pt"})
    got = pkg.safetensors_to_blob(path, shape_to_cfg(pkg, shape, 0))
    want = torch.from_numpy(blob).to(td).float().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_gpt2_errors_name_the_tensor(tmp_path):
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 33, 0)
    sd = {k: v.contiguous() for k, v in _gpt2_hf(shape, blob).state_dict().items() if k != "lm_head.weight"}
    cfg = shape_to_cfg(pkg, shape, 0)
    missing = dict(sd)
    del missing["transformer.h.1.mlp.c_fc.bias"]
    p1 = str(tmp_path / "missing.safetensors")
    st_torch.save_file(missing, p1)
    with pytest.raises(pkg.Gpt2Error, match="h.1.mlp.c_fc.bias"):
        pkg.safetensors_to_blob(p1, cfg)
    wrong = dict(sd)
    wrong["transformer.h.0.attn.c_attn.weight"] = wrong["transformer.h.0.attn.c_attn.weight"].T.contiguous()
    p2 = str(tmp_path / "wrong.safetensors")
    st_torch.save_file(wrong, p2)
    with pytest.raises(pkg.Gpt2Error, match="c_attn.weight has shape"):
        pkg.safetensors_to_blob(p2, cfg)
    p3 = str(tmp_path / "garbage.safetensors")
    with open(p3, "wb") as f:
        f.write(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json at all}")
    with pytest.raises(pkg.Gpt2Error, match="header"):
        pkg.safetensors_to_blob(p3, cfg)
    with pytest.raises(pkg.Gpt2Error, match="cannot open"):
        pkg.safetensors_to_blob(str(tmp_path / "absent.safetensors"), cfg)


def test_bert_save_pretrained_and_legacy_names(tmp_path):
    """BertModel.save_pretrained reads back bit for bit; so does a BertForPreTraining-style file
    ("bert." prefix, LayerNorm gamma / beta, an extra cls head)."""
    shape = O.BERT_TINY
    blob = O.bert_seeded_blob(shape, 34, 1)
    model = _bert_hf(shape, blob)
    model.save_pretrained(tmp_path, safe_serialization=True)
    cfg = _bert_cfg(shape)
    got = pkg.bert.safetensors_to_blob(str(tmp_path / "model.safetensors"), cfg)
    assert np.array_equal(got.view(np.uint32), blob.view(np.uint32))
    legacy = {}
    for k, v in model.state_dict().items():
        if "LayerNorm.weight" in k:
            k = k.replace("LayerNorm.weight", "LayerNorm.gamma")
        elif "LayerNorm.bias" in k:
            k = k.replace("LayerNorm.bias", "LayerNorm.beta")
        legacy["bert." + k] = v.contiguous()
    legacy["cls.predictions.bias"] = torch.zeros(shape.vocab_size)
    p = str(tmp_path / "legacy.safetensors")
    st_torch.save_file(legacy, p)
    got = pkg.bert.safetensors_to_blob(p, cfg)
    assert np.array_equal(got.view(np.uint32), blob.view(np.uint32))
