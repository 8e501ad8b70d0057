"""Programmatic dependent launch of the few-token chain (the GEMV and short /
decode attention kernels start while the kernel before them finishes and
prefetch their weights, then wait for it): results must be bit-identical to
plain launches, for the FP32 and BF16 few-token forwards (plain, captured and
replayed) and for greedy decoding.  The launch mode is fixed per process, so
each mode runs in a child process (tests/pdl_worker.py)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from helpers import HERE

pytestmark = pytest.mark.gpu


def _run(tmp_path, pdl):
    path = os.path.join(tmp_path, f"pdl{pdl}.npz")
    env = dict(os.environ)
    env.pop("GPT2_PDL", None)
    if not pdl:
        env["GPT2_PDL"] = "0"
    r = subprocess.run(["timeout", "-k", "10", "300", sys.executable, os.path.join(HERE, "pdl_worker.py"), path],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return dict(np.load(path))


def test_programmatic_launches_match_plain_launches(tmp_path):
    on, off = _run(str(tmp_path), True), _run(str(tmp_path), False)
    assert sorted(on) == sorted(off)
    for k in on:
        assert np.array_equal(on[k], off[k]), k
    for d in (0, 1):  # graph capture and replay give the plain launch's logits
        assert np.array_equal(on[f"fwd_d{d}_0"], on[f"fwd_d{d}_2"])
    assert np.isfinite(on["fwd_d0_0"]).all() and np.isfinite(on["fwd_d1_0"]).all()
