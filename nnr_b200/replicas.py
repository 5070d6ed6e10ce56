"""Batch-sharded replicas: the multi-GPU form of the hot path.

The path shards by image: each rank runs the whole network on its own batch
of images (no data-path collective). What the ranks share is host-side:
which images a rank takes, one seeded model built once and handed to the
others, and the job's time as the maximum over ranks (a collective on the
timing tensor only). These helpers take the process group as an argument so
that they run under NCCL on the GPU box and under gloo on the CPU.
"""
from __future__ import annotations

import os
import pickle
from pathlib import Path
from typing import Callable, List, Sequence


def shard_offset(rank: int, per_rank: int) -> int:
    """First image index of a rank's batch: rank r takes images
    [r * per_rank, (r + 1) * per_rank) of the job's global batch."""
    return rank * per_rank


def build_once(build: Callable[[], object], key: str, rank: int, world: int, barrier: Callable[[], None]):
    """Rank 0 builds the object (a seeded model) and the other ranks load the
    same bytes; the file is named by `key` (unique per job) in TMPDIR."""
    if world == 1:
        return build()
    path = Path(os.environ.get("TMPDIR", "/tmp")) / f"nnrcu_{key}.pkl"
    if rank == 0:
        obj = build()
        tmp = path.with_suffix(".tmp")
        tmp.write_bytes(pickle.dumps(obj))
        os.replace(tmp, path)
    barrier()
    return pickle.loads(path.read_bytes())


def max_over_ranks(values: Sequence[float], world: int, dist=None, device=None) -> List[float]:
    """Element-wise maximum over the ranks of per-rank times (the job ends
    when its slowest rank does)."""
    if world == 1 or dist is None:
        return [float(v) for v in values]
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_rate(per_rank: int, world: int, ms_per_step: float) -> float:
    """Whole-job images per second: every rank's batch per step over the
    (max-over-ranks) step time."""
    return world * per_rank / (ms_per_step / 1e3)
