"""Helpers shared by the tests: package / oracle loading, fixtures, comparisons."""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")


def load_pkg():
    """Imports the mlir-learning_b200 package (its directory name is not a Python identifier)."""
    name = "mlir_learning_b200"
    if name in sys.modules:
        return sys.modules[name]
    path = os.path.join(ROOT, "mlir-learning_b200", "__init__.py")
    spec = importlib.util.spec_from_file_location(name, path, submodule_search_locations=[os.path.dirname(path)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import oracle as O
    return O


def golden_files():
    """GPT-2 fixtures."""
    return sorted(f for f in glob.glob(os.path.join(GOLDEN, "*.npz")) if not os.path.basename(f).startswith("bert_"))


def bert_golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "bert_*.npz")))


def load_bert_golden(path):
    O = load_oracle()
    z = dict(np.load(path))
    s = [int(x) for x in z["shape"]]
    shape = O.BertShape(s[0], s[1], s[2], s[3], s[4], s[5], float(z["eps"]), s[6])
    return shape, z


def load_golden(path):
    O = load_oracle()
    z = dict(np.load(path))
    s = [int(x) for x in z["shape"]]
    shape = O.ModelShape(*s, float(z["eps"]))
    return shape, z


def shape_to_cfg(pkg, shape, dtype):
    return pkg.Gpt2Config(shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                          shape.n_positions, shape.layer_norm_eps, dtype)


def attendable_rows(mask: np.ndarray) -> np.ndarray:
    """[B, S] bool: query row has at least one attendable key (k <= q with mask[k] != 0)."""
    return np.cumsum(mask != 0, axis=1) > 0


# Stated parity bounds of the reduced-precision paths, as fractions of the oracle's max |logit| (one
# calibration run on a B200 measured |logit - oracle| / max |logit| at every logit of every comparison
# the GPU tests make; the figures are beside each constant).
#   MAX_REL: every logit within this bound.
#   TOP5_BOUND_REL: the per-logit error bound under which top-5 identity is required: at every
#   position whose oracle top-5 logits each lead the next one (1st over 2nd ... 5th over 6th) by
#   more than twice this bound, the same five ids in the same order.
BF16_MAX_REL = 0.015          # observed max 4.8e-3 (tiny) .. 1.15e-2 (GPT-2 small, random gains)
BF16_TOP5_BOUND_REL = 0.005   # the 99.9th percentile on the headline workload: 5.4e-3, 5.9e-3
FP8_DEQ_MAX_REL = 0.025       # FP8-weight kernels vs the oracle on the dequantized weights: max 1.7e-2 (48 layers)
FP8_F32_MAX_REL = 0.15        # vs the FP32 weights (quantization included): max 6.7e-2 (2 layers), 9.7e-2 (48)
PARITY_LOG = os.environ.get("GPT2_PARITY_LOG")  # JSON lines of every report, when set


def top5_check(label, ref, got, *, max_rel, bound_rel=None, min_checked=None, min_top1=None, min_overlap=None):
    """Holds reduced-precision logits `got` to the oracle's `ref` ([..., V]).

    Always: max |got - ref| <= max_rel * max |ref|.  With bound_rel: top-5 identity at every
    position checkable under the stated bound bound_rel * max |ref| (oracle.top5_report), and, where
    given, floors on the checkable fraction of positions (min_checked), the unconditional top-1
    agreement over all positions (min_top1) and the mean size of the top-5 set intersection
    (min_overlap, out of 5).  The report is printed (and appended to $GPT2_PARITY_LOG)."""
    import json
    O = load_oracle()
    scale = float(np.abs(ref).max())
    rep = O.top5_report(ref, got, (bound_rel if bound_rel is not None else max_rel) * scale)
    rep.update(label=label, scale=scale, max_rel=rep["max_err"] / scale, bound_rel=bound_rel)
    print(f"{label}: max|diff| {rep['max_err']:.4g} (rel {rep['max_rel']:.3g} of {scale:.3g}); "
          f"top-5 checkable {rep['checked']}/{rep['total']} ({rep['checked'] / rep['total']:.3f}) under rel bound "
          f"{bound_rel}, identical {rep['identical']}; top-1 {rep['top1']:.4f}; top-5 overlap {rep['overlap']:.3f}; "
          f"logits past the bound {rep['exceed']:.2e}")
    if PARITY_LOG:
        with open(PARITY_LOG, "a") as f:
            f.write(json.dumps(rep) + "\n")
    assert rep["max_err"] <= max_rel * scale, (label, rep["max_rel"], max_rel)
    if bound_rel is not None:
        assert rep["identical"] == rep["checked"], (label, rep["identical"], rep["checked"])
    if min_checked is not None:
        assert rep["checked"] >= min_checked * rep["total"], (label, rep["checked"], rep["total"], min_checked)
    if min_top1 is not None:
        assert rep["top1"] >= min_top1, (label, rep["top1"], min_top1)
    if min_overlap is not None:
        assert rep["overlap"] >= min_overlap, (label, rep["overlap"], min_overlap)
    return rep


def attention_ref(torch, qkv, mask, B, S, H, causal=True):
    """float64 restatement of the oracle's attention semantics."""
    D = H * 64
    x = qkv.double().view(B, S, 3, H, 64)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    s = q @ k.transpose(-1, -2) * 0.125
    ok = torch.ones(S, S, dtype=torch.bool, device=qkv.device)
    if causal:
        ok = ok.tril()
    ok = ok[None, None]
    if mask is not None:
        ok = ok & (mask != 0)[:, None, None, :]
    s = s.masked_fill(~ok, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = p @ v
    none = ~ok.any(-1)  # [B,1|H,S]
    mean_v = v.mean(dim=2, keepdim=True).expand_as(o)
    o = torch.where(none[..., None].expand_as(o), mean_v, o)
    return o.transpose(1, 2).reshape(B * S, D)
