"""Batch sharding across ranks (one process per GPU) and the step-time
reduction used by the benchmark.

The decode path partitions by batch row: rank r owns rows [start, start +
count) of the global batch with its own tiers, and runs its layers with no
collective on the data path (the output of a layer stays on the rank that
computed it).  The only cross-rank traffic is bookkeeping: the max of the
ranks' step times and small host objects.
"""

from __future__ import annotations

import torch


def batch_shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, rows) of `rank`'s shard: contiguous, sizes differing by at
    most one, every row owned by exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device: torch.device | str | None = None) -> float:
    """Maximum of a per-rank scalar (e.g. a step time) over the process group;
    the value itself when torch.distributed is not initialised."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_objects(obj) -> list:
    """Every rank's `obj` (in rank order); [obj] without a process group."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


__all__ = ["batch_shard", "gather_objects", "max_over_ranks"]
