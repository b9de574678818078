"""Helpers shared by the GPU tests: numpy <-> torch with exact bits."""

from __future__ import annotations

import numpy as np
import torch

from oracle.numerics import from_bits, to_bits

TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
NAME_DT = {v: k for k, v in TORCH_DT.items()}


def t_from_bits(b: np.ndarray, dt: str, device="cuda") -> torch.Tensor:
    """Storage bits (uint16/uint32) -> torch tensor of dtype dt on device."""
    if dt == "f32":
        return torch.from_numpy(np.ascontiguousarray(b).view(np.float32)).to(device)
    t = torch.from_numpy(np.ascontiguousarray(b).astype(np.uint16).view(np.int16))
    return t.view(TORCH_DT[dt]).to(device)


def t_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def t_vals(t: torch.Tensor) -> np.ndarray:
    """Values as float32 numpy (exact for fp16/bf16)."""
    return t.detach().float().cpu().numpy()


def np_to_dt_tensor(x: np.ndarray, dt: str, device="cuda") -> torch.Tensor:
    """float32 values already representable in dt -> exact torch tensor."""
    return t_from_bits(to_bits(np.asarray(x, dtype=np.float32), dt), dt, device)


def seeded_outliers(shape, seed: int, dt: str, n_out=4, mult=8.0) -> np.ndarray:
    """N(0,1) with `n_out` outlier channels per head scaled by `mult`, rounded to dt."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    H, D = shape[1], shape[-1]
    for h in range(H):
        ch = rng.permutation(D)[:n_out]
        x[:, h, :, ch] *= mult
    return from_bits(to_bits(x, dt), dt) if dt != "f32" else x


def dtype_ulp(x: np.ndarray, dt: str) -> np.ndarray:
    """Spacing of the dtype's representable values at |x|."""
    mb = {"f16": 10, "bf16": 7, "f32": 23}[dt]
    tiny = {"f16": 2.0 ** -24, "bf16": 2.0 ** -133, "f32": 2.0 ** -149}[dt]
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 1e-300)))
    return np.maximum(2.0 ** (e - mb), tiny)


def assert_attn_close(out: np.ndarray, ref: np.ndarray, dt: str, atol: float, ulps: float = 1.0,
                      additive: bool = False) -> float:
    """Attention parity criterion: |out - ref| <= max(atol, 1 ulp of the output
    dtype at |ref|) element-wise.  atol is the north-star tolerance (2e-3 fp16,
    1e-2 bf16); the ulp term is the unavoidable rounding of a result stored in
    the dtype (two correctly computed outputs can land one ulp apart when the
    exact value is near a rounding boundary, which exceeds atol once |ref| >= 4
    in fp16 or >= 2 in bf16).  Returns the worst err / limit."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    u = ulps * dtype_ulp(ref, dt)
    lim = atol + u if additive else np.maximum(atol, u)
    ratio = np.abs(out - ref) / lim
    worst = float(ratio.max()) if ratio.size else 0.0
    maxabs = float(np.abs(out - ref).max()) if ratio.size else 0.0
    print(f"[attn {dt}] max|out-ref| = {maxabs:.3e} (north-star atol {atol:g}), worst err/limit {worst:.3f}")
    assert worst <= 1.0, f"max |out-ref| {np.abs(out - ref).max():.3e}, worst err/limit {worst:.3f}"
    return worst
