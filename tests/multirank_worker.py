"""Worker for tests/test_gpu_multirank.py, launched with torchrun: every rank
runs the BF16 forward of its shard of the batch on its own GPU through the C
ABI, NCCL gathers the logits to rank 0, and rank 0 compares them bit for bit
with a single-GPU forward of the whole batch.  Exit code 0 = equal."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
import bench  # noqa: E402
from helpers import load_oracle, load_pkg, shape_to_cfg  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    pkg, O = load_pkg(), load_oracle()
    shape = O.GPT2_SMALL
    pkg.init(shape_to_cfg(pkg, shape, pkg.DTYPE_BF16), local)
    pkg.init_seeded(1234, 0)
    Bg, S, V, LD = 4 * world, 512, shape.vocab_size, 50304
    ids_all = pkg.seeded_ids(Bg, S, 1234, V)
    r0, r1 = bench.shard_rows(Bg, world, rank)
    ids = torch.from_numpy(np.ascontiguousarray(ids_all[r0:r1])).cuda()
    logits = torch.empty((r1 - r0) * S, LD, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    pkg.forward_device(ids.data_ptr(), None, r1 - r0, S, logits.data_ptr(), LD, st)
    torch.cuda.synchronize()
    assert pkg.status() == 0
    glist = [torch.empty_like(logits) for _ in range(world)] if rank == 0 else None
    dist.gather(logits, glist, dst=0)
    ok = torch.ones(1, device="cuda")
    if rank == 0:
        full_ids = torch.from_numpy(ids_all).cuda()
        full = torch.empty(Bg * S, LD, device="cuda")
        pkg.forward_device(full_ids.data_ptr(), None, Bg, S, full.data_ptr(), LD, st)
        torch.cuda.synchronize()
        got = torch.cat(glist)
        ok[0] = float(torch.equal(got[:, :V], full[:, :V]))
        print(f"rank0: gathered {tuple(got.shape)} equal={bool(ok.item())}", flush=True)
    dist.broadcast(ok, src=0)
    pkg.shutdown()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() == 1.0 else 1)


if __name__ == "__main__":
    main()
