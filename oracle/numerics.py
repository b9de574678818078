"""Rounding helpers: emulate torch's fp16/bf16 per-op arithmetic in numpy.

torch evaluates an elementwise fp16/bf16 op in fp32 and rounds the result to
the storage type once (round-to-nearest-even).  ``rnd(x, dt)`` performs that
rounding on a float32 array and returns float32 holding the rounded values.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import numpy as np


def f16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest float16 (RNE, numpy's conversion) -> float32."""
    with np.errstate(over="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (RNE on the top 16 bits) -> float32; NaN kept."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def rnd(x: np.ndarray, dt: str) -> np.ndarray:
    if dt == "f16":
        return f16_round(x)
    if dt == "bf16":
        return bf16_round(x)
    if dt == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dt)


def eps(dt: str) -> np.float32:
    """torch's clamp(min=1e-8) threshold as seen in `dt`."""
    return np.float32(rnd(np.float32(1e-8), dt))


def to_bits(x: np.ndarray, dt: str) -> np.ndarray:
    """Raw storage bits of dtype-valued float32 data (for bit comparisons)."""
    x = np.asarray(x, dtype=np.float32)
    if dt == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dt == "bf16":
        return (x.view(np.uint32) >> 16).astype(np.uint16)
    return x.view(np.uint32)


def from_bits(b: np.ndarray, dt: str) -> np.ndarray:
    b = np.asarray(b)
    if dt == "f16":
        return b.astype(np.uint16).view(np.float16).astype(np.float32)
    if dt == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.astype(np.uint32).view(np.float32)
