"""Multi-GPU batch sharding with the NCCL logits gather, on
every GPU of the box: launches tests/multirank_worker.py with torchrun; the
gathered logits must equal a single-GPU forward of the whole batch bit for
bit.  Skipped on boxes with fewer than two GPUs."""
import os
import subprocess
import sys

import pytest

from helpers import HERE

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two or more GPUs")
def test_sharded_forward_gathered_equals_single_gpu():
    n = _gpus()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, "multirank_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "equal=True" in out.stdout
