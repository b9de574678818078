"""Pluggable quantisation backends (the reference's ``fade/backends.py``).

``QuantBackend`` is the reference's protocol (``fade/backends.py:36-58``):
``compress_k/v(x) -> dict[str, Tensor]``, ``decompress_k/v(d, dtype)`` and a
``name``.  The built-in backends run the sm_100a kernels:

* ``SymmetricINT4Backend`` ("int4", "symmetric_int4"): per-channel K /
  per-token V INT4, bit-packed (``fade_b200.quant``);
* ``RotatedINT4Backend`` ("rotated", "rotated_int4"): seeded orthogonal
  rotation then 2/3/4-bit quantisation (``fade_b200.rotated_quant``); the
  fused decode kernel reads its 2- and 4-bit codes directly.

``TurboQuantBackend`` ("turbo", "turboquant") wraps the third-party
``turboquant-kv`` package exactly as the reference does; that package is not
part of this build, so using it raises the reference's ImportError.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

import torch
from torch import Tensor

from fade_b200.quant import dequant_int4, quant_k_int4, quant_v_int4


@runtime_checkable
class QuantBackend(Protocol):
    """Protocol for K/V cache quantisation backends."""

    def compress_k(self, k: Tensor) -> dict[str, Tensor]: ...

    def decompress_k(self, compressed: dict[str, Tensor], dtype: torch.dtype) -> Tensor: ...

    def compress_v(self, v: Tensor) -> dict[str, Tensor]: ...

    def decompress_v(self, compressed: dict[str, Tensor], dtype: torch.dtype) -> Tensor: ...

    @property
    def name(self) -> str: ...


@dataclass
class SymmetricINT4Backend:
    """Per-channel K, per-token V, bit-packed INT4."""

    @property
    def name(self) -> str:
        return "symmetric_int4"

    def compress_k(self, k: Tensor) -> dict[str, Tensor]:
        packed, scale = quant_k_int4(k)
        return {"packed": packed, "scale": scale}

    def decompress_k(self, compressed: dict[str, Tensor], dtype: torch.dtype = torch.float16) -> Tensor:
        return dequant_int4(compressed["packed"], compressed["scale"], dtype=dtype)

    def compress_v(self, v: Tensor) -> dict[str, Tensor]:
        packed, scale = quant_v_int4(v)
        return {"packed": packed, "scale": scale}

    def decompress_v(self, compressed: dict[str, Tensor], dtype: torch.dtype = torch.float16) -> Tensor:
        return dequant_int4(compressed["packed"], compressed["scale"], dtype=dtype)


@dataclass
class RotatedINT4Backend:
    """Rotation before quantisation (``bits`` 2, 3 or 4; seeded R per device)."""

    head_dim: int = 64
    bits: int = 4
    seed: int = 42
    _R: dict = field(default_factory=dict, init=False, repr=False)

    @property
    def name(self) -> str:
        return f"rotated_int{self.bits}"

    def rotation(self, device: torch.device | None = None) -> Tensor:
        """The [head_dim, head_dim] fp32 rotation on ``device``."""
        from fade_b200.rotated_quant import _random_orthogonal

        key = torch.device(device) if device is not None else torch.device("cpu")
        if key not in self._R:
            self._R[key] = _random_orthogonal(self.head_dim, self.seed).to(key)
        return self._R[key]

    def compress_k(self, k: Tensor) -> dict[str, Tensor]:
        from fade_b200.rotated_quant import rotated_quant_k

        packed, scale = rotated_quant_k(k, self.rotation(k.device), bits=self.bits)
        return {"packed": packed, "scale": scale}

    def decompress_k(self, compressed: dict[str, Tensor], dtype: torch.dtype = torch.float16) -> Tensor:
        from fade_b200.rotated_quant import rotated_dequant_k

        p = compressed["packed"]
        return rotated_dequant_k(p, compressed["scale"], self.rotation(p.device), bits=self.bits, dtype=dtype)

    def compress_v(self, v: Tensor) -> dict[str, Tensor]:
        from fade_b200.rotated_quant import rotated_quant_v

        packed, scale = rotated_quant_v(v, self.rotation(v.device), bits=self.bits)
        return {"packed": packed, "scale": scale}

    def decompress_v(self, compressed: dict[str, Tensor], dtype: torch.dtype = torch.float16) -> Tensor:
        from fade_b200.rotated_quant import rotated_dequant_v

        p = compressed["packed"]
        return rotated_dequant_v(p, compressed["scale"], self.rotation(p.device), bits=self.bits, dtype=dtype)


@dataclass
class TurboQuantBackend:
    """Placeholder for the reference's optional ``turboquant-kv`` backend.

    TurboQuant is a third-party quantiser outside this library's hot path; the
    name stays registered (``"turbo"`` / ``"turboquant"``) so configurations
    that mention it fail the same way as the reference does when the optional
    package is absent: with an ImportError on first use.
    """

    head_dim: int = 128
    bits: float = 4
    device: str | None = None

    @property
    def name(self) -> str:
        return f"turboquant_{self.bits}bit"

    def _unavailable(self, *args, **kwargs):
        raise ImportError(
            "TurboQuantBackend requires turboquant-kv. Install with: pip install fade-kv[turbo]"
        )

    compress_k = decompress_k = compress_v = decompress_v = _unavailable


_BACKENDS: dict[str, type] = {
    "symmetric_int4": SymmetricINT4Backend,
    "int4": SymmetricINT4Backend,
    "rotated_int4": RotatedINT4Backend,
    "rotated": RotatedINT4Backend,
    "turbo": TurboQuantBackend,
    "turboquant": TurboQuantBackend,
}


def get_backend(name: str = "int4", **kwargs) -> QuantBackend:
    """Backend by name; keyword arguments go to the backend's constructor
    (those it does not take are ignored, as in the reference)."""
    cls = _BACKENDS.get(name.lower())
    if cls is None:
        raise ValueError(f"Unknown quant backend {name!r}. Available: {list(_BACKENDS.keys())}")
    if cls is SymmetricINT4Backend:
        return cls()
    fields = {k for k, f in cls.__dataclass_fields__.items() if f.init and not k.startswith("_")}
    return cls(**{k: v for k, v in kwargs.items() if k in fields})


__all__ = [
    "QuantBackend",
    "RotatedINT4Backend",
    "SymmetricINT4Backend",
    "TurboQuantBackend",
    "get_backend",
]
