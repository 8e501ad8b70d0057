"""The reference's own host program, src/gpt/gpt2_call.cpp, compiled unchanged
against libgpt2_b200.so (oracle/Makefile target ref-host), run on the GPU.

It calls gpt2_decoder on ids [464, 3139, 286, 4881, 318] with an all-ones mask
(src/gpt/gpt2_call.cpp:54-64) and prints the first 10 logits of the last
position (%14.6f) and the top-5 (%.4f).  With the default seeded weights
(GPT2_SEED 1234, FP32) that is the case of tests/golden/gpt2_small_refcall.npz,
so the printed numbers are checked against transformers' logits."""
import os
import re
import subprocess

import numpy as np
import pytest

from helpers import GOLDEN, ROOT

pytestmark = pytest.mark.gpu
BIN = os.path.join(ROOT, "oracle", "_ref", "gpt2_call")


@pytest.mark.skipif(not os.path.exists(BIN), reason="oracle/_ref/gpt2_call is built only where the reference "
                                                     "sources exist (make -C oracle ref-host)")
def test_reference_host_program_runs_unchanged():
    env = dict(os.environ, GPT2_SEED="1234", GPT2_DTYPE="f32")
    out = subprocess.run([BIN], capture_output=True, text=True, env=env, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    z = np.load(os.path.join(GOLDEN, "gpt2_small_refcall.npz"))
    last = z["logits"][0, -1]
    vals = [float(v) for v in re.findall(r"vocab\[\s*\d+\] =\s*(-?\d+\.\d+)", out.stdout)]
    assert len(vals) == 10, out.stdout
    assert np.abs(np.array(vals) - last[:10]).max() <= 1e-4 + 1e-6
    top = [(int(i), float(v)) for i, v in re.findall(r"token_id=\s*(\d+)\s+logit=(-?\d+\.\d+)", out.stdout)]
    assert [i for i, _ in top] == list(z["top5_idx"][0, -1])
    assert np.abs(np.array([v for _, v in top]) - z["top5_val"][0, -1]).max() <= 1e-4 + 5e-5
