"""Work partition of the decode step across ranks (one process per GPU).

The units of work (sequence b, kv head h, layer) are independent, and a
rank's KV cache never moves.  Two partitions:

* ``"heads"`` (the default for more than one GPU): rank r owns kv heads
  [r*Hkv/N, (r+1)*Hkv/N) of every sequence, with the g = Hq/Hkv query heads
  that read them.  After each layer the ranks all-gather their attention
  outputs over NCCL (the only data-path collective), so every rank ends the
  layer holding out[B, Hq, D] for the whole batch.  At 8 GPUs and Hkv = 8 this
  is one kv head per GPU.
* ``"batch"``: rank r owns a contiguous slice of the batch with all heads;
  a layer's output stays on the rank that computed it (no collective).

``ShardPlan`` gives a rank its shapes; ``assemble_heads`` is the permutation
that turns the rank-major gathered buffer into head order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def batch_shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, rows) of `rank`'s shard: contiguous, sizes differing by at
    most one, every row owned by exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class ShardPlan:
    mode: str            # "heads" or "batch"
    world: int
    rank: int
    batch: int           # rows of the batch this rank holds
    batch0: int          # its first row in the global batch
    n_kv_heads: int      # kv heads this rank holds
    kv_head0: int        # its first kv head
    n_q_heads: int       # query heads this rank computes

    @property
    def gathers(self) -> bool:
        return self.mode == "heads" and self.world > 1


def shard_plan(mode: str, world: int, rank: int, global_batch: int, n_q_heads: int, n_kv_heads: int) -> ShardPlan:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_q_heads % n_kv_heads:
        raise ValueError("n_q_heads must be a multiple of n_kv_heads")
    g = n_q_heads // n_kv_heads
    if mode == "heads":
        if n_kv_heads % world:
            raise ValueError(f"{n_kv_heads} kv heads do not split over {world} ranks")
        hk = n_kv_heads // world
        return ShardPlan("heads", world, rank, global_batch, 0, hk, rank * hk, hk * g)
    if mode == "batch":
        b0, nb = batch_shard(global_batch, world, rank)
        return ShardPlan("batch", world, rank, nb, b0, n_kv_heads, 0, n_q_heads)
    raise ValueError(f"unknown shard mode {mode!r}")


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """[N, B, Hq/N, ...] (rank-major all-gather of per-rank outputs) ->
    [B, Hq, ...] in head order: rank r's head j is global head r*Hq/N + j."""
    N, B, hq = gathered.shape[:3]
    return gathered.transpose(0, 1).reshape(B, N * hq, *gathered.shape[3:])


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


__all__ = ["ShardPlan", "assemble_heads", "batch_shard", "gather_objects", "max_over_ranks", "shard_plan"]
