"""RoPE schemes: cos/sin tables for the eviction re-RoPE (``fade/rope.py``).

The re-RoPE kernel (``fade_rerope_gather``) takes float32 cos/sin tables; to
cancel the model's own rotary embedding exactly they are built the way the
reference builds them (``fade/rope.py:72-93``): inverse frequencies in fp32,
``angle = position * inv_freq`` duplicated over both halves, cos/sin in fp32
and, unless the model dtype is bf16, rounded through the model dtype.  Table
construction is a few small torch ops on the cache's device.

Schemes (same names and parameters as the reference): ``Vanilla``,
``LinearScaled``, ``Llama3`` (``llama3`` / ``longrope`` scaling), ``NtkAware``
(``ntk`` / ``dynamic``), ``Yarn``, ``Proportional`` (partial rotation),
``MRope`` (text-only: shared axes), ``NoRope`` (identity tables).
"""

from __future__ import annotations

import math
import warnings
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch
from torch import Tensor

DEFAULT_ROPE_THETA: float = 10000.0
DEFAULT_FACTOR: float = 1.0
DEFAULT_LOW_FREQ_FACTOR: float = 1.0
DEFAULT_HIGH_FREQ_FACTOR: float = 4.0
DEFAULT_ORIGINAL_MAX_POS: int = 8192
DEFAULT_YARN_BETA_FAST: float = 32.0
DEFAULT_YARN_BETA_SLOW: float = 1.0


def _base_inv_freq(rot_dim: int, denom: int, theta: float, device) -> Tensor:
    exps = torch.arange(0, rot_dim, 2, dtype=torch.float32, device=device) / denom
    return 1.0 / (theta ** exps)


def _tables(angles: Tensor, model_dtype: torch.dtype, round_trip: bool) -> tuple[Tensor, Tensor]:
    c, s = angles.cos(), angles.sin()
    if round_trip:
        c, s = c.to(model_dtype).float(), s.to(model_dtype).float()
    return c[None, None], s[None, None]


@dataclass
class RopeScheme:
    """Standard RoPE; subclasses change the inverse frequencies or positions."""

    theta: float = DEFAULT_ROPE_THETA
    head_dim: int = 64
    _inv: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    def _compute_inv_freq(self, device) -> Tensor:
        return _base_inv_freq(self.head_dim, self.head_dim, self.theta, device)

    def inv_freq(self, device) -> Tensor:
        """``[head_dim // 2]`` inverse frequencies (cached per device)."""
        key = torch.device(device)
        if key not in self._inv:
            self._inv[key] = self._compute_inv_freq(key)
        return self._inv[key]

    def _angles(self, positions: Tensor, device) -> Tensor:
        f = positions.to(device).float()[:, None] * self.inv_freq(device)[None, :]
        return torch.cat((f, f), dim=-1)

    def compute_cos_sin(self, positions: Tensor, device, model_dtype: torch.dtype = torch.float16):
        """(cos, sin), float32, broadcastable to ``[1, 1, S, head_dim]``."""
        return _tables(self._angles(positions, device), model_dtype, model_dtype != torch.bfloat16)

    @property
    def is_rope(self) -> bool:
        return True


@dataclass
class Vanilla(RopeScheme):
    """Standard RoPE (Qwen2, Mistral, Phi-3, Gemma-2, ...)."""


@dataclass
class LinearScaled(RopeScheme):
    """Positions divided by ``factor``."""

    factor: float = DEFAULT_FACTOR

    def compute_cos_sin(self, positions, device, model_dtype=torch.float16):
        f = (positions.to(device).float() / self.factor)[:, None] * self.inv_freq(device)[None, :]
        return _tables(torch.cat((f, f), dim=-1), model_dtype, True)


@dataclass
class Llama3(RopeScheme):
    """Llama-3.1 band-wise interpolation of the inverse frequencies."""

    factor: float = DEFAULT_FACTOR
    low_freq_factor: float = DEFAULT_LOW_FREQ_FACTOR
    high_freq_factor: float = DEFAULT_HIGH_FREQ_FACTOR
    original_max_position_embeddings: int = DEFAULT_ORIGINAL_MAX_POS

    def _compute_inv_freq(self, device):
        base = _base_inv_freq(self.head_dim, self.head_dim, self.theta, device)
        ctx = float(self.original_max_position_embeddings)
        wl = 2.0 * math.pi / base
        t = (ctx / wl - self.low_freq_factor) / (self.high_freq_factor - self.low_freq_factor)
        mid = base * (1 - t) / self.factor + base * t
        low_band = wl > ctx / self.low_freq_factor
        high_band = wl < ctx / self.high_freq_factor
        return torch.where(high_band, base, torch.where(low_band, base / self.factor, mid))


@dataclass
class NtkAware(RopeScheme):
    """Base frequency scaled by ``factor``."""

    factor: float = DEFAULT_FACTOR

    def _compute_inv_freq(self, device):
        return _base_inv_freq(self.head_dim, self.head_dim, self.theta * self.factor, device)


@dataclass
class Yarn(RopeScheme):
    """YaRN: per-dimension ramp between interpolated and NTK frequencies."""

    factor: float = DEFAULT_FACTOR
    beta_fast: float = DEFAULT_YARN_BETA_FAST
    beta_slow: float = DEFAULT_YARN_BETA_SLOW
    original_max_position_embeddings: int = DEFAULT_ORIGINAL_MAX_POS

    def _compute_inv_freq(self, device):
        base = _base_inv_freq(self.head_dim, self.head_dim, self.theta, device)
        ntk = _base_inv_freq(self.head_dim, self.head_dim, self.theta * self.factor, device)
        idx = torch.arange(base.shape[0], dtype=torch.float32, device=device)
        denom = 2 * math.pi * self.original_max_position_embeddings
        lo = self.beta_fast * self.head_dim / denom
        hi = self.beta_slow * self.head_dim / denom
        ramp = ((idx - lo) / (hi - lo)).clamp(0.0, 1.0)
        return (1.0 - ramp) * base / self.factor + ramp * ntk


@dataclass
class Proportional(RopeScheme):
    """Partial rotation with head_dim-based exponents; unrotated pairs get
    inverse frequency 0 (cos 1, sin 0)."""

    partial_rotary_factor: float = 1.0

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def _compute_inv_freq(self, device):
        n_rot = self.rotary_dim // 2
        inv = _base_inv_freq(2 * n_rot, self.head_dim, self.theta, device)
        pad = self.head_dim // 2 - n_rot
        if pad > 0:
            inv = torch.cat([inv, torch.zeros(pad, dtype=torch.float32, device=device)])
        return inv


@dataclass
class MRope(RopeScheme):
    """Multi-resolution RoPE; for text the three position axes coincide, so
    the tables are vanilla RoPE over ``rotary_dim`` (zero angles beyond)."""

    partial_rotary_factor: float = 1.0
    mrope_section: list | None = None

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def _compute_inv_freq(self, device):
        return _base_inv_freq(self.rotary_dim, self.rotary_dim, self.theta, device)

    def compute_cos_sin(self, positions, device, model_dtype=torch.float16):
        f = positions.to(device).float()[:, None] * self.inv_freq(device)[None, :]
        a = torch.cat((f, f), dim=-1)
        if self.rotary_dim < self.head_dim:
            a = torch.cat([a, torch.zeros(a.shape[0], self.head_dim - self.rotary_dim, device=device)], dim=-1)
        return _tables(a, model_dtype, True)


@dataclass
class NoRope(RopeScheme):
    """Models without rotary embeddings: identity tables."""

    def compute_cos_sin(self, positions, device, model_dtype=torch.float16):
        S = positions.shape[0]
        return (torch.ones(1, 1, S, self.head_dim, dtype=torch.float32, device=device),
                torch.zeros(1, 1, S, self.head_dim, dtype=torch.float32, device=device))

    @property
    def is_rope(self) -> bool:
        return False


def _head_dim_of(cfg, head_dim):
    if head_dim is not None:
        return head_dim
    hd = getattr(cfg, "head_dim", None)
    if hd is None:
        hd = getattr(cfg, "hidden_size", 64) // getattr(cfg, "num_attention_heads", 1)
    return hd


def _scheme_from_params(rp: dict, head_dim: int, fallback_theta: float) -> RopeScheme:
    theta = float(rp.get("rope_theta", fallback_theta))
    kind = str(rp.get("rope_type", rp.get("type", "default"))).lower()
    prf = float(rp.get("partial_rotary_factor", 1.0))
    if kind == "proportional" or (kind in ("", "default") and prf < 1.0):
        return Proportional(theta=theta, head_dim=head_dim, partial_rotary_factor=prf)
    if kind in ("", "default"):
        return Vanilla(theta=theta, head_dim=head_dim)
    rest = {k: v for k, v in rp.items() if k not in ("rope_theta", "rope_type", "type")}
    shim = SimpleNamespace(rope_theta=theta, rope_scaling={"type": kind, **rest}, hidden_size=head_dim,
                           num_attention_heads=1)
    return extract_rope_scheme(shim, head_dim=head_dim)


def extract_rope_schemes_per_layer(cfg, head_dim: int | None = None) -> dict | None:
    """``{layer_type: scheme}`` for configs with per-layer-type RoPE
    (nested ``rope_parameters``), else None."""
    rp = getattr(cfg, "rope_parameters", None)
    if not isinstance(rp, dict) or not isinstance(next(iter(rp.values()), None), dict):
        return None
    hd = _head_dim_of(cfg, head_dim)
    fb = float(getattr(cfg, "rope_theta", DEFAULT_ROPE_THETA))
    return {k: _scheme_from_params(v, hd, fb) for k, v in rp.items() if isinstance(v, dict)}


def extract_rope_scheme(cfg, head_dim: int | None = None) -> RopeScheme:
    """RoPE scheme of a HF config (``rope_theta`` / ``rope_scaling`` or the
    5.x ``rope_parameters`` layout); the full-attention scheme for per-layer
    configs."""
    per_layer = extract_rope_schemes_per_layer(cfg, head_dim)
    if per_layer is not None:
        return per_layer.get("full_attention", next(iter(per_layer.values())))
    rp = getattr(cfg, "rope_parameters", None)
    theta = getattr(cfg, "rope_theta", None)
    if theta is None and isinstance(rp, dict):
        theta = rp.get("rope_theta")
    theta = float(DEFAULT_ROPE_THETA if theta is None else theta)
    hd = _head_dim_of(cfg, head_dim)
    if getattr(cfg, "alibi", False) or getattr(cfg, "model_type", "") in ("bloom", "mpt"):
        return NoRope(theta=theta, head_dim=hd)
    section = rp.get("mrope_section") if isinstance(rp, dict) else None
    if section is None:
        section = getattr(cfg, "mrope_section", None)
    if section is not None:
        prf = float(rp.get("partial_rotary_factor", 1.0)) if isinstance(rp, dict) else 1.0
        return MRope(theta=theta, head_dim=hd, partial_rotary_factor=prf, mrope_section=list(section))
    rs = getattr(cfg, "rope_scaling", None)
    if not isinstance(rs, dict):
        return Vanilla(theta=theta, head_dim=hd)
    kind = str(rs.get("type", rs.get("rope_type", ""))).lower()
    prf = float(rs.get("partial_rotary_factor", 1.0))
    if kind == "proportional" or (kind in ("", "default") and prf < 1.0):
        return Proportional(theta=theta, head_dim=hd, partial_rotary_factor=prf)
    if kind in ("", "default"):
        return Vanilla(theta=theta, head_dim=hd)
    factor = float(rs.get("factor", 1.0))
    orig = int(rs.get("original_max_position_embeddings",
                      getattr(cfg, "original_max_position_embeddings", DEFAULT_ORIGINAL_MAX_POS)))
    if kind == "linear":
        return LinearScaled(theta=theta, head_dim=hd, factor=factor)
    if kind in ("llama3", "longrope"):
        return Llama3(theta=theta, head_dim=hd, factor=factor,
                      low_freq_factor=float(rs.get("low_freq_factor", DEFAULT_LOW_FREQ_FACTOR)),
                      high_freq_factor=float(rs.get("high_freq_factor", DEFAULT_HIGH_FREQ_FACTOR)),
                      original_max_position_embeddings=orig)
    if kind in ("ntk", "dynamic"):
        return NtkAware(theta=theta, head_dim=hd, factor=factor)
    if kind == "yarn":
        return Yarn(theta=theta, head_dim=hd, factor=factor,
                    beta_fast=float(rs.get("beta_fast", DEFAULT_YARN_BETA_FAST)),
                    beta_slow=float(rs.get("beta_slow", DEFAULT_YARN_BETA_SLOW)),
                    original_max_position_embeddings=orig)
    warnings.warn(f"Unknown rope_scaling type {kind!r}; falling back to vanilla RoPE.", RuntimeWarning,
                  stacklevel=2)
    return Vanilla(theta=theta, head_dim=hd)


__all__ = [
    "LinearScaled",
    "Llama3",
    "MRope",
    "NoRope",
    "NtkAware",
    "Proportional",
    "RopeScheme",
    "Vanilla",
    "Yarn",
    "extract_rope_scheme",
    "extract_rope_schemes_per_layer",
]
