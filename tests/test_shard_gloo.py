"""Multi-rank host logic on CPU: two gloo ranks shard a batch and reduce a
step time the way bench.py does on NCCL ranks."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_batch_shard_partitions():
    from fade_b200.shard import batch_shard

    for B in (1, 7, 16, 128):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                s, n = batch_shard(B, world, r)
                rows.extend(range(s, s + n))
            assert rows == list(range(B))
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fade_b200.shard import batch_shard, gather_objects, max_over_ranks

        start, n = batch_shard(32, world, rank)
        step_ms = 1.0 + rank                       # rank-dependent "step time"
        q.put((rank, start, n, max_over_ranks(step_ms), gather_objects(f"bus{rank}")))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(r, s, n) for r, s, n, _, _ in res] == [(0, 0, 16), (1, 16, 16)]
    assert all(m == 2.0 for _, _, _, m, _ in res)          # max over ranks
    assert all(g == ["bus0", "bus1"] for *_, g in res)


def test_kv_head_plan_covers_heads():
    """Every (b, kv head) of the batch is owned by exactly one rank; each rank
    holds the g query heads of its kv heads."""
    from fade_b200.shard import shard_plan

    for world in (1, 2, 4, 8):
        owned = []
        for r in range(world):
            p = shard_plan("heads", world, r, 128, 64, 8)
            assert p.batch == 128 and p.n_q_heads == p.n_kv_heads * 8 and p.gathers == (world > 1)
            owned.extend(range(p.kv_head0, p.kv_head0 + p.n_kv_heads))
        assert owned == list(range(8))
    with pytest.raises(ValueError):
        shard_plan("heads", 3, 0, 16, 32, 8)


def _heads_rank(rank: int, world: int, port: int, q) -> None:
    """One rank: attention (float64 oracle) of its kv heads' query heads, then
    the all-gather + permutation bench.py applies to every layer's output."""
    import numpy as np

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fade_b200.shard import assemble_heads, shard_plan
        from oracle.attention import sdpa

        B, Hq, Hkv, S, D = 3, 8, 4, 50, 16
        rng = np.random.default_rng(0)               # identical global tensors on every rank
        qg = rng.standard_normal((B, Hq, 1, D))
        kg = rng.standard_normal((B, Hkv, S, D))
        vg = rng.standard_normal((B, Hkv, S, D))
        p = shard_plan("heads", world, rank, B, Hq, Hkv)
        h0, g = p.kv_head0, Hq // Hkv
        local = sdpa(qg[:, h0 * g:(h0 + p.n_kv_heads) * g], kg[:, h0:h0 + p.n_kv_heads],
                     vg[:, h0:h0 + p.n_kv_heads])
        t = torch.from_numpy(local).contiguous()
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        full = assemble_heads(torch.stack(parts))
        q.put((rank, np.abs(full.numpy() - sdpa(qg, kg, vg)).max()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_kv_head_shard_gather():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_heads_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r for r, _ in res] == [0, 1]
    assert all(err == 0.0 for _, err in res)     # same float64 math, only regrouped
