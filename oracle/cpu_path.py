"""The reference's per-step CPU decode path, restated -- TEST AND CPU-BASELINE USE ONLY.

What the reference pays per layer per decode step on the CPU (fade/cache.py:
update -> _materialize 683-808 -> torch.cat 699, with the INT4 middle's
dequantised copy cached between reassignments 810-842), followed by the HF
SDPA it feeds (transformers sdpa_attention.py:40-62, enable_gqa):

    K = cat(sink_k, dequant(middle_k), recent_k); V likewise
    out = scaled_dot_product_attention(q, K, V, enable_gqa=True)

Used by bench.py's ``--impl reference`` arm and its ``cpu_baseline`` leg.  The
product never imports this module.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def build_layer_state(B: int, Hkv: int, D: int, n_sink: int, n_mid: int, n_rec: int, dtype: torch.dtype,
                      seed: int = 0) -> dict:
    """Synthetic tier state of one layer in the reference's cached form: FP sink
    and recent tensors plus the middle already dequantised (cache_dequant=True)."""
    g = torch.Generator().manual_seed(seed)

    def rnd(n):
        x = torch.randn(B, Hkv, n, D, generator=g)
        return x.to(dtype)

    return {
        "sink_k": rnd(n_sink), "sink_v": rnd(n_sink),
        "mid_k": rnd(n_mid), "mid_v": rnd(n_mid),
        "rec_k": rnd(n_rec), "rec_v": rnd(n_rec),
    }


def reference_layer_step(q: torch.Tensor, st: dict) -> torch.Tensor:
    K = torch.cat([st["sink_k"], st["mid_k"], st["rec_k"]], dim=-2)
    V = torch.cat([st["sink_v"], st["mid_v"], st["rec_v"]], dim=-2)
    return F.scaled_dot_product_attention(q, K, V, enable_gqa=True)


def time_layer_steps(B: int, Hq: int, Hkv: int, D: int, n_sink: int, n_mid: int, n_rec: int,
                     dtype: torch.dtype, steps: int, warmup: int, threads: int) -> list[float]:
    """Seconds per single-layer step (list of `steps` samples) on `threads` CPU threads."""
    torch.set_num_threads(threads)
    st = build_layer_state(B, Hkv, D, n_sink, n_mid, n_rec, dtype)
    g = torch.Generator().manual_seed(1)
    q = torch.randn(B, Hq, 1, D, generator=g).to(dtype)
    for _ in range(warmup):
        reference_layer_step(q, st)
    out = []
    for _ in range(steps):
        t0 = time.perf_counter()
        reference_layer_step(q, st)
        out.append(time.perf_counter() - t0)
    return out
