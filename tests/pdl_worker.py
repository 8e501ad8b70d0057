"""Worker for tests/test_gpu_pdl.py, run as a child process (the launch mode
is read from the environment once per process, GPT2_PDL=0 meaning plain
launches): GPT-2 small with seeded weights on cuda:0, the few-token forward
(FP32 B1 x S5, the reference host program's call, and BF16 B2 x S8, each run
plainly, then captured and replayed as a CUDA graph) and greedy KV-cache
decoding in BF16 (B 1 and 16).  Writes every output to the .npz named by
argv[1]."""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from helpers import load_pkg  # noqa: E402


def main():
    torch.cuda.set_device(0)
    pkg = load_pkg()
    st = torch.cuda.current_stream().cuda_stream
    out = {}
    for dtype, B, S in ((pkg.DTYPE_F32, 1, 5), (pkg.DTYPE_BF16, 2, 8)):
        pkg.init(pkg.gpt2_small(dtype), 0)
        pkg.init_seeded(1234, 0)
        ids = torch.from_numpy(pkg.seeded_ids(B, S, 77, 50257)).cuda()
        logits = torch.empty(B * S, 50260, device="cuda")
        for i in range(3):  # plain, capture + launch, replay
            pkg.forward_device(ids.data_ptr(), None, B, S, logits.data_ptr(), 50260, st)
            torch.cuda.synchronize()
            out[f"fwd_d{dtype}_{i}"] = logits[:, :50257].cpu().numpy()
        assert pkg.status() == 0
        if dtype == pkg.DTYPE_BF16:
            for Bd in (1, 16):
                prompt = pkg.seeded_ids(Bd, 12, 78, 50257)
                out[f"gen_B{Bd}"] = pkg.generate(prompt, 6)
            assert pkg.status() == 0
        pkg.shutdown()
    np.savez(sys.argv[1], **out)


if __name__ == "__main__":
    main()
