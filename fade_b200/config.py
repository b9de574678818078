"""FADE tuning configuration (the reference's ``fade/config.py:33-157``).

``FadeConfig`` keeps the reference's field names, defaults, validation
messages, presets and ``to_cache_kwargs()`` so existing callers
(``create_tiered_cache(model, config=FadeConfig.safe())``) work unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Literal

DEFAULT_N_SINK: int = 4
DEFAULT_RECENT_WINDOW: int = 64
DEFAULT_INT2_GROUP_SIZE: int = 64
DEFAULT_REASSIGN_EVERY: int = 64
DEFAULT_PREFILL_TRACK_LIMIT: int = 1024

EvictionPolicy = Literal["h2o", "ema", "position", "learned"]
Phase = Literal["1a", "2"]
QuantBits = Literal[4, 2]
QuantBackendName = Literal["int4", "turbo"]

_POLICIES = ("h2o", "ema", "position", "learned")


@dataclass(frozen=True)
class FadeConfig:
    """Validated cache configuration.

    phase "1a": INT4 middle, nothing evicted (``int4_budget`` must be None);
    phase "2": budget-bounded eviction with re-RoPE (some budget > 0).
    ``middle_k_bits`` / ``middle_v_bits`` select 4- or 2-bit middle tiers;
    ``quant_backend`` names a backend of ``fade_b200.backends.get_backend``.
    """

    phase: Phase = "1a"
    n_sink: int = DEFAULT_N_SINK
    recent_window: int = DEFAULT_RECENT_WINDOW
    int4_budget: int | None = None
    int2_budget: int = 0
    eviction_policy: EvictionPolicy = "h2o"
    reassign_every: int = DEFAULT_REASSIGN_EVERY
    prefill_track_limit: int = DEFAULT_PREFILL_TRACK_LIMIT
    int2_group_size: int = DEFAULT_INT2_GROUP_SIZE
    middle_k_bits: QuantBits = 4
    middle_v_bits: QuantBits = 4
    quant_backend: QuantBackendName = "int4"
    _extras: dict = field(default_factory=dict, repr=False)

    def __post_init__(self) -> None:
        checks = [
            (self.n_sink < 0, f"n_sink must be >= 0, got {self.n_sink}"),
            (self.recent_window < 0, f"recent_window must be >= 0, got {self.recent_window}"),
            (self.int4_budget is not None and self.int4_budget < 0,
             f"int4_budget must be >= 0 or None, got {self.int4_budget}"),
            (self.int2_budget < 0, f"int2_budget must be >= 0, got {self.int2_budget}"),
            (self.reassign_every < 1, f"reassign_every must be >= 1, got {self.reassign_every}"),
            (self.int2_group_size < 1, f"int2_group_size must be >= 1, got {self.int2_group_size}"),
            (self.phase == "1a" and self.int4_budget is not None,
             "phase='1a' requires int4_budget=None (no eviction); "
             f"got int4_budget={self.int4_budget}"),
            (self.phase == "2" and self.int4_budget is None and self.int2_budget == 0,
             "phase='2' requires at least one of int4_budget / int2_budget > 0"),
            (self.eviction_policy not in _POLICIES, f"unknown eviction_policy: {self.eviction_policy!r}"),
            (self.middle_k_bits not in (4, 2), f"middle_k_bits must be 4 or 2, got {self.middle_k_bits}"),
            (self.middle_v_bits not in (4, 2), f"middle_v_bits must be 4 or 2, got {self.middle_v_bits}"),
        ]
        for bad, msg in checks:
            if bad:
                raise ValueError(msg)

    # presets -------------------------------------------------------------
    @classmethod
    def safe(cls) -> FadeConfig:
        """INT4 middle, no eviction (~3-4x KV compression)."""
        return cls(phase="1a", n_sink=4, recent_window=64)

    @classmethod
    def balanced(cls) -> FadeConfig:
        """H2O eviction with a 400-token INT4 budget (~5x)."""
        return cls(phase="2", n_sink=4, recent_window=64, int4_budget=400, int2_budget=0, eviction_policy="h2o")

    @classmethod
    def aggressive(cls) -> FadeConfig:
        """H2O eviction with a 200-token INT4 budget and a 32-token window (~7-8x)."""
        return cls(phase="2", n_sink=4, recent_window=32, int4_budget=200, int2_budget=0, eviction_policy="h2o")

    def with_overrides(self, **kwargs) -> FadeConfig:
        """Copy with fields replaced (validated again)."""
        return replace(self, **kwargs)

    def to_cache_kwargs(self) -> dict:
        """Keyword arguments for ``TieredKVCache(**config.to_cache_kwargs())``."""
        return {
            "n_sink": self.n_sink,
            "recent_window": self.recent_window,
            "int4_budget": self.int4_budget,
            "int2_budget": self.int2_budget,
            "middle_k_bits": self.middle_k_bits,
            "middle_v_bits": self.middle_v_bits,
            "quant_backend": self.quant_backend,
        }


__all__ = [
    "DEFAULT_INT2_GROUP_SIZE",
    "DEFAULT_N_SINK",
    "DEFAULT_PREFILL_TRACK_LIMIT",
    "DEFAULT_REASSIGN_EVERY",
    "DEFAULT_RECENT_WINDOW",
    "EvictionPolicy",
    "FadeConfig",
    "Phase",
    "QuantBackendName",
    "QuantBits",
]
