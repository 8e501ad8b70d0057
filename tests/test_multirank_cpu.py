"""The batch-sharded multi-rank path on CPU, world size 2 over gloo: the shard
arithmetic bench.py uses, the max-over-ranks timing, and that sharding the
batch over ranks and gathering the per-rank logits to rank 0 reproduces the
single-process forward (sequences never mix, so no data-path collective is
needed).  The per-rank forward here is the oracle, standing in for each GPU."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from helpers import ROOT, load_oracle

import sys
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_shard_rows():
    assert bench.shard_rows(64, 1, 0) == (0, 64)
    assert [bench.shard_rows(64, 8, r) for r in range(8)] == [(8 * r, 8 * r + 8) for r in range(8)]
    with pytest.raises(ValueError):
        bench.shard_rows(64, 3, 0)
    with pytest.raises(ValueError):
        bench.shard_rows(64, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O = load_oracle()
    shape = O.GPT2_TINY
    blob = O.seeded_blob(shape, 5, 1)
    ids = O.token_ids(4, 19, 5, shape.vocab_size)
    mask = np.ones_like(ids)
    mask[2, :3] = 0
    r0, r1 = bench.shard_rows(4, world, rank)
    local = torch.from_numpy(O.forward(shape, blob, ids[r0:r1], mask[r0:r1]))
    glist = [torch.empty_like(local) for _ in range(world)] if rank == 0 else None
    dist.gather(local, glist, dst=0)
    t = bench.max_over_ranks(float(rank + 1), dist, "cpu")
    if rank == 0:
        full = O.forward(shape, blob, ids, mask)
        np.save(os.path.join(out_dir, "gathered.npy"), torch.cat(glist).numpy())
        np.save(os.path.join(out_dir, "full.npy"), full)
        np.save(os.path.join(out_dir, "tmax.npy"), np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_forward_equals_single_process(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    gathered = np.load(tmp_path / "gathered.npy")
    full = np.load(tmp_path / "full.npy")
    assert gathered.shape == full.shape
    assert np.array_equal(gathered, full)
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0
