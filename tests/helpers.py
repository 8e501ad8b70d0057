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


def top5_agreement(ref: np.ndarray, got: np.ndarray, bound: float | None = None):
    """Top-5 identity over the positions whose reference top-5 is separated (between adjacent
    top-5 entries and between the 5th and 6th logit) by more than twice the error at that
    position (the max |got - ref| over its row; or `bound` when given).  Returns
    (checked positions, agreeing positions, total positions)."""
    r = ref.reshape(-1, ref.shape[-1])
    g = got.reshape(-1, got.shape[-1])
    idx = np.argsort(-r, axis=1, kind="stable")[:, :6]
    vals = np.take_along_axis(r, idx, axis=1)
    gaps = vals[:, :5] - vals[:, 1:6]
    row_err = np.abs(g - r).max(axis=1) if bound is None else np.full(r.shape[0], bound)
    separated = (gaps > 2 * row_err[:, None]).all(axis=1)
    gidx = np.argsort(-g, axis=1, kind="stable")[:, :5]
    same = (gidx == idx[:, :5]).all(axis=1)
    return int(separated.sum()), int((same & separated).sum()), r.shape[0]


def top1_fraction(ref: np.ndarray, got: np.ndarray) -> float:
    r = ref.reshape(-1, ref.shape[-1])
    g = got.reshape(-1, got.shape[-1])
    return float((r.argmax(axis=1) == g.argmax(axis=1)).mean())
