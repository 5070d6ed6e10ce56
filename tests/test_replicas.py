"""The multi-GPU form of the path (batch-sharded replicas) on two gloo ranks
on the CPU: image shards are disjoint and cover the global batch, the seeded
model built by rank 0 reaches every rank unchanged, and the job's time is the
maximum over ranks, as bench.py uses them under NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nnr_b200 import replicas


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tmpdir, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), TMPDIR=tmpdir)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        barrier = dist.barrier
        # rank 0 builds; the others must see exactly its object
        obj = replicas.build_once(lambda: {"w": np.arange(10) * (rank + 1), "built_by": rank}, f"t{port}", rank,
                                  world, barrier)
        # per-rank times: the job's time is the slowest rank's
        mx = replicas.max_over_ranks([1.0 + rank, 5.0 - rank], world, dist)
        off = replicas.shard_offset(rank, 32)
        out[rank] = (obj["built_by"], obj["w"].tolist(), mx, off)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    world, port = 2, _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, port, str(tmp_path), out), nprocs=world, join=True)
    assert sorted(out.keys()) == [0, 1]
    for r in range(world):
        built_by, w, mx, off = out[r]
        assert built_by == 0 and w == list(range(10))
        assert mx == [2.0, 5.0]
        assert off == 32 * r
    # shards of the global batch: disjoint, covering [0, world * 32)
    cover = sorted(i for r in range(world) for i in range(out[r][3], out[r][3] + 32))
    assert cover == list(range(world * 32))


def test_single_rank_is_local():
    assert replicas.max_over_ranks([3.0, 4.0], 1) == [3.0, 4.0]
    assert replicas.build_once(lambda: 7, "x", 0, 1, lambda: None) == 7
    assert replicas.job_rate(32, 8, 0.5) == pytest.approx(8 * 32 / 0.5e-3)
