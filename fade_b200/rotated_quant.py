"""Rotation-based quantisation (reference ``fade/rotated_quant.py``) on sm_100a.

``x_rot = x @ R^T`` then symmetric quantisation at 2/3/4 bits in fp32: K with a
per-channel scale over the sequence, V with a per-token scale; the scale is
cast to the input dtype.  Codes are packed like the reference (INT4 nibbles,
2-bit four per byte, 3-bit unpacked int8).  The rotation accumulates in fp32
in a fixed sequential order; the reference's CPU matmul may round a rotated
value differently by an ulp, which can move a code by one at a rounding
boundary (rare; the scales and all other codes match).
"""

from __future__ import annotations

import torch
from torch import Tensor

from fade_b200 import _lib
from fade_b200.quant import _pack_int2_last_dim, _pack_int4_last_dim, _unpack_int2_last_dim, _unpack_int4_last_dim

DEFAULT_SEED: int = 42
EPS: float = 1e-8

_BIT_PARAMS: dict[int, tuple[int, int]] = {4: (-8, 7), 3: (-4, 3), 2: (-2, 1)}


def _random_orthogonal(dim: int, seed: int = DEFAULT_SEED) -> Tensor:
    """Seeded random orthogonal matrix via QR (``fade/rotated_quant.py:91-96``).

    Generated on the host with torch's CPU generator, so the matrix is the same
    bits as the reference's for the same (dim, seed); it is a parameter, not
    part of the decode path."""
    gen = torch.Generator().manual_seed(seed)
    M = torch.randn(dim, dim, generator=gen)
    Q, _ = torch.linalg.qr(M)
    return Q


def _packed_last(D: int, bits: int) -> int:
    return D // 2 if bits == 4 else (D // 4 if bits == 2 else D)


def _rot(x: Tensor, R: Tensor, bits: int, kind: int) -> tuple[Tensor, Tensor]:
    if bits not in _BIT_PARAMS:
        raise KeyError(bits)
    if x.dim() != 4:
        raise ValueError(f"expected [B, H, S, D], got shape {tuple(x.shape)}")
    B, H, S, D = x.shape
    if bits == 4 and D % 2:
        raise ValueError(f"last dim must be even for INT4 packing, got {D}")
    if bits == 2 and D % 4:
        raise ValueError(f"last dim must be divisible by 4 for INT2 packing, got {D}")
    dev = _lib.require_cuda(x)
    Rd = R.to(device=dev, dtype=torch.float32).contiguous()
    packed = torch.empty(B, H, S, _packed_last(D, bits), dtype=torch.uint8 if bits != 3 else torch.int8, device=dev)
    scale = torch.empty((B, H, 1, D) if kind == 0 else (B, H, S, 1), dtype=x.dtype, device=dev)
    ws = torch.empty(max(B * H * D * 4, 16), dtype=torch.uint8, device=dev) if kind == 0 else None
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_rotated_quant(
            x.data_ptr(), _lib.dtype_code(x.dtype), _lib.view4(x), Rd.data_ptr(), bits, kind,
            packed.data_ptr(), scale.data_ptr(), _lib.ptr(ws), 0 if ws is None else ws.numel(), st
        ),
        "rotated_quant",
    )
    return packed, scale


def rotated_quant_k(k: Tensor, R: Tensor, bits: int = 4) -> tuple[Tensor, Tensor]:
    """``fade/rotated_quant.py:106-131``: (packed, scale [B,H,1,D])."""
    return _rot(k, R, bits, 0)


def rotated_quant_v(v: Tensor, R: Tensor, bits: int = 4) -> tuple[Tensor, Tensor]:
    """``fade/rotated_quant.py:148-173``: (packed, scale [B,H,S,1])."""
    return _rot(v, R, bits, 1)


def _rot_deq(packed: Tensor, scale: Tensor, R: Tensor, bits: int, dtype: torch.dtype, mode: int) -> Tensor:
    dev = _lib.require_cuda(packed, scale)
    B, H, S, P = packed.shape
    D = P * 2 if bits == 4 else (P * 4 if bits == 2 else P)
    Rd = R.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(B, H, S, D, dtype=dtype, device=dev)
    sc = scale.to(dtype).contiguous()
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_rotated_dequant(packed.contiguous().data_ptr(), bits, sc.data_ptr(), mode, Rd.data_ptr(),
                                         _lib.dtype_code(dtype), B, H, S, D, out.data_ptr(), st),
        "rotated_dequant",
    )
    return out


def rotated_dequant_k(packed: Tensor, scale: Tensor, R: Tensor, bits: int = 4,
                      dtype: torch.dtype = torch.float16) -> Tensor:
    """``fade/rotated_quant.py:134-145``."""
    return _rot_deq(packed, scale, R, bits, dtype, 0)


def rotated_dequant_v(packed: Tensor, scale: Tensor, R: Tensor, bits: int = 4,
                      dtype: torch.dtype = torch.float16) -> Tensor:
    """``fade/rotated_quant.py:176-187``."""
    return _rot_deq(packed, scale, R, bits, dtype, 1)


def _pack(q: Tensor, bits: int) -> Tensor:
    if bits == 4:
        return _pack_int4_last_dim(q)
    if bits == 2:
        return _pack_int2_last_dim(q)
    return q.to(torch.int8)


def _unpack(packed: Tensor, bits: int) -> Tensor:
    if bits == 4:
        return _unpack_int4_last_dim(packed)
    if bits == 2:
        return _unpack_int2_last_dim(packed)
    return packed.to(torch.int8)


__all__ = ["rotated_dequant_k", "rotated_dequant_v", "rotated_quant_k", "rotated_quant_v"]
