"""Batch sharding for one process per GPU.

Batch rows of the contextualizer are independent (every sum in the forward
runs over the context or the features of one batch row), so a multi-GPU run
gives each rank a contiguous slice of the batch and runs the single-GPU path
on it: no data crosses GPUs. Collectives are used only outside timed regions,
for the maximum of the per-rank times and for gathering rows to rank 0 for
verification.

The process-group plumbing here is plain ``torch.distributed``; it runs over
NCCL on GPUs and over gloo on CPU ranks (the tests use the latter).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

__all__ = ['rank_env', 'shard_bounds', 'shard', 'max_over_ranks', 'gather_to_rank0']


def rank_env() -> tuple[int, int, int]:
    """(world size, global rank, local rank) from the torchrun environment."""
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    return world, rank, local


def shard_bounds(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Half-open batch range [start, stop) of `rank` out of `world` ranks.

    The batch must split evenly: ranks that hold different amounts of work
    would make the max-over-ranks time measure the largest shard only.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} is not in a world of {world}')
    if global_batch < 0 or global_batch % world:
        raise ValueError(f'global batch {global_batch} does not split over {world} ranks')
    per = global_batch // world
    return rank * per, (rank + 1) * per


def shard(t: torch.Tensor, world: int, rank: int, dim: int = 0) -> torch.Tensor:
    """The view of `t` that `rank` owns along `dim` (no copy)."""
    start, stop = shard_bounds(t.shape[dim], world, rank)
    return t.narrow(dim, start, stop - start)


def _active() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def max_over_ranks(x: float, device: torch.device | None = None) -> float:
    """Maximum of a per-rank scalar over all ranks (identity without a group)."""
    if not _active():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(t: torch.Tensor) -> list[torch.Tensor] | None:
    """Every rank's `t` (same shape and dtype on all ranks), on rank 0.

    Returns the list in rank order on rank 0 and None elsewhere; without a
    process group it returns [t].
    """
    if not _active():
        return [t]
    t = t.contiguous()
    rank = dist.get_rank()
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())] if rank == 0 else None
    dist.gather(t, out, dst=0)
    return out
