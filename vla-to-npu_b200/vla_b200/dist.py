"""Observation partitioning across GPUs (one process per GPU).

The SmolVLA hot path has no cross-observation data dependence, so a batch is
split into contiguous per-rank shards, each rank runs the whole chunk forward
on its shard with its own weight replica, and nothing crosses GPUs on the data
path.  ``gather_actions`` collects the per-rank action chunks afterwards (off
the timed path) with one all-gather, for callers that want them in one place.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch


def shard_bounds(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of rank's observations: contiguous, sizes differing by at most 1."""
    if world <= 0 or not 0 <= rank < world or global_batch < 0:
        raise ValueError(f"bad shard request: batch={global_batch} rank={rank} world={world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(obs: Dict[str, torch.Tensor], rank: int, world: int) -> Dict[str, torch.Tensor]:
    n = next(iter(obs.values())).shape[0]
    a, b = shard_bounds(n, rank, world)
    return {k: v[a:b] for k, v in obs.items()}


def gather_actions(local: torch.Tensor, global_batch: int, group=None) -> torch.Tensor:
    """All-gather per-rank action chunks [b_r, chunk, dim] into [global_batch, chunk, dim]
    (rank order = observation order).  Shards are padded to the largest shard."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    biggest = shard_bounds(global_batch, 0, world)
    pad = biggest[1] - biggest[0]
    buf = torch.zeros((pad,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    out = []
    for r, p in enumerate(parts):
        a, b = shard_bounds(global_batch, r, world)
        out.append(p[: b - a])
    return torch.cat(out, dim=0)
