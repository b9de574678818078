"""Numpy restatement of the eviction re-RoPE -- TEST INFRASTRUCTURE ONLY.

fade/cache.py:283-311 (_rotate_half, _apply_rope, _inverse_rope) and the
evicting branch of apply_tier_assignment, fade/cache.py:914-935: un-RoPE at
the old positions, keep the survivors, re-RoPE at 0..n_kept-1.  Each torch op
there is a separate fp32 elementwise op, restated one-to-one here.
cos/sin tables are inputs (the RopeScheme's, fade/rope.py:72-93).
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import rnd


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rope(k: np.ndarray, cos: np.ndarray, sin: np.ndarray, dt: str) -> np.ndarray:
    k = np.asarray(k, dtype=np.float32)
    a = (k * cos).astype(np.float32)
    b = (rotate_half(k) * sin).astype(np.float32)
    return rnd((a + b).astype(np.float32), dt)


def inverse_rope(k: np.ndarray, cos: np.ndarray, sin: np.ndarray, dt: str) -> np.ndarray:
    k = np.asarray(k, dtype=np.float32)
    a = (k * cos).astype(np.float32)
    b = (rotate_half(k) * sin).astype(np.float32)
    return rnd((a - b).astype(np.float32), dt)


def rerope_gather(k: np.ndarray, keep: np.ndarray, cos_old, sin_old, cos_new, sin_new, dt: str) -> np.ndarray:
    """k [B,H,S,D]; keep int [n]; cos_old [S,D]; cos_new [n,D] -> [B,H,n,D]."""
    pre = inverse_rope(k, cos_old, sin_old, dt)
    kept = pre[..., keep, :]
    return apply_rope(kept, cos_new, sin_new, dt)


def vanilla_cos_sin(positions: np.ndarray, head_dim: int, theta: float, dt: str):
    """Vanilla RoPE tables in fp32 with the fp16 round trip the reference applies
    for non-bf16 model dtypes (fade/rope.py:38-46, 72-93).  Note: numpy's cos/sin
    can differ from torch's by an ulp; tests that need exact tables load them
    from the golden fixtures."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)))).astype(np.float32)
    freqs = positions.astype(np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float32)
    c, s = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    if dt != "bf16":
        c, s = rnd(c, "f16"), rnd(s, "f16")
    return c, s
