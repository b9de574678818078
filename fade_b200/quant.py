"""Quantisation primitives for the K/V cache, on sm_100a kernels.

Same API, storage formats and bit-exact results as the reference's
``fade/quant.py`` (fade-kv 1.1.0), computed by ``libfade_sm100.so``:

* K: per-channel symmetric INT4 (absmax over the sequence axis),
  ``fade/quant.py:61-75``.
* V: per-token symmetric INT4 (absmax over head_dim), ``fade/quant.py:78-92``.
* INT4 packing: byte ``d`` = (code ``2d`` in the high nibble, code ``2d+1`` in
  the low nibble), two's complement, ``fade/quant.py:26-58``.
* Grouped INT2 along the sequence axis with per-(group, channel) scales,
  ``fade/quant.py:95-176``; returned as int8 codes like the reference, and
  available 4-codes-per-byte packed for the cache (``quant_int2_grouped_packed``).

The rounding sequence is the reference's: every fp16/bf16 op is an fp32 op
rounded once to the dtype, and ``qmax / absmax`` is torch's ``__rtruediv__``,
i.e. ``reciprocal(absmax)`` rounded, times ``qmax``, rounded.
"""

from __future__ import annotations

import torch
from torch import Tensor

from fade_b200 import _lib

# --- knobs (same names and values as the reference) ------------------------- #
INT4_MIN: int = -8
INT4_MAX: int = 7
INT2_MIN: int = -2
INT2_MAX: int = 1
EPS: float = 1e-8
DEFAULT_INT2_GROUP_SIZE: int = 64


def _contig_out(shape, dtype, device) -> Tensor:
    return torch.empty(shape, dtype=dtype, device=device)


def _pack_int4_last_dim(q_int8: Tensor) -> Tensor:
    """Pack pairs of INT4 values into uint8 bytes along the last dim
    (reference ``fade/quant.py:26-43``)."""
    if q_int8.shape[-1] % 2 != 0:
        raise ValueError(f"last dim must be even for INT4 packing, got {q_int8.shape[-1]}")
    dev = _lib.require_cuda(q_int8)
    q = q_int8.to(torch.int8).contiguous()
    D = q.shape[-1]
    rows = q.numel() // D if D else 0
    out = _contig_out((*q.shape[:-1], D // 2), torch.uint8, dev)
    st = _lib.bind(dev)
    _lib.check(_lib.load().fade_pack_codes(q.data_ptr(), rows, D, 4, out.data_ptr(), st), "pack_int4")
    return out


def _unpack_int4_last_dim(packed: Tensor) -> Tensor:
    """Inverse of ``_pack_int4_last_dim`` (reference ``fade/quant.py:46-58``)."""
    dev = _lib.require_cuda(packed)
    p = packed.contiguous()
    Dh = p.shape[-1]
    rows = p.numel() // Dh if Dh else 0
    out = _contig_out((*p.shape[:-1], Dh * 2), torch.int8, dev)
    st = _lib.bind(dev)
    _lib.check(_lib.load().fade_unpack_codes(p.data_ptr(), rows, Dh * 2, 4, out.data_ptr(), st), "unpack_int4")
    return out


def _pack_int2_last_dim(q: Tensor) -> Tensor:
    """Pack 4 INT2 codes per byte (reference ``fade/rotated_quant.py:35-48``)."""
    if q.shape[-1] % 4 != 0:
        raise ValueError(f"last dim must be divisible by 4 for INT2 packing, got {q.shape[-1]}")
    dev = _lib.require_cuda(q)
    qc = q.to(torch.int8).contiguous()
    D = qc.shape[-1]
    rows = qc.numel() // D if D else 0
    out = _contig_out((*qc.shape[:-1], D // 4), torch.uint8, dev)
    st = _lib.bind(dev)
    _lib.check(_lib.load().fade_pack_codes(qc.data_ptr(), rows, D, 2, out.data_ptr(), st), "pack_int2")
    return out


def _unpack_int2_last_dim(packed: Tensor) -> Tensor:
    """Inverse of ``_pack_int2_last_dim`` (reference ``fade/rotated_quant.py:51-69``)."""
    dev = _lib.require_cuda(packed)
    p = packed.contiguous()
    Dq = p.shape[-1]
    rows = p.numel() // Dq if Dq else 0
    out = _contig_out((*p.shape[:-1], Dq * 4), torch.int8, dev)
    st = _lib.bind(dev)
    _lib.check(_lib.load().fade_unpack_codes(p.data_ptr(), rows, Dq * 4, 2, out.data_ptr(), st), "unpack_int2")
    return out


def _quant_int4(x: Tensor, per_channel: bool) -> tuple[Tensor, Tensor]:
    if x.dim() != 4:
        raise ValueError(f"expected [B, H, S, D], got shape {tuple(x.shape)}")
    B, H, S, D = x.shape
    if D % 2 != 0:
        raise ValueError(f"last dim must be even for INT4 packing, got {D}")
    dev = _lib.require_cuda(x)
    dt = _lib.dtype_code(x.dtype)
    packed = _contig_out((B, H, S, D // 2), torch.uint8, dev)
    scale = _contig_out((B, H, 1, D) if per_channel else (B, H, S, 1), x.dtype, dev)
    st = _lib.bind(dev)
    fn = _lib.load().fade_quant_int4_k if per_channel else _lib.load().fade_quant_int4_v
    _lib.check(fn(x.data_ptr(), dt, _lib.view4(x), packed.data_ptr(), scale.data_ptr(), st),
               "quant_int4")
    return packed, scale


def quant_k_int4(k: Tensor) -> tuple[Tensor, Tensor]:
    """Per-channel symmetric INT4 for K, bit-packed.

    Returns ``(packed [B,H,S,D/2] uint8, scale [B,H,1,D] k.dtype)``, bit-identical
    to ``fade/quant.py:61-75``.
    """
    return _quant_int4(k, per_channel=True)


def quant_v_int4(v: Tensor) -> tuple[Tensor, Tensor]:
    """Per-token symmetric INT4 for V, bit-packed.

    Returns ``(packed [B,H,S,D/2] uint8, scale [B,H,S,1] v.dtype)``, bit-identical
    to ``fade/quant.py:78-92``.
    """
    return _quant_int4(v, per_channel=False)


def _quant_int2(x: Tensor, group_size: int, want_i8: bool, want_packed: bool):
    B, H, S, D = x.shape
    if S % group_size != 0:
        raise ValueError(f"S={S} must be divisible by group_size={group_size}")
    if want_packed and D % 4 != 0:
        raise ValueError(f"last dim must be divisible by 4 for INT2 packing, got {D}")
    dev = _lib.require_cuda(x)
    dt = _lib.dtype_code(x.dtype)
    G = S // group_size
    q8 = _contig_out((B, H, S, D), torch.int8, dev) if want_i8 else None
    qp = _contig_out((B, H, S, D // 4), torch.uint8, dev) if want_packed else None
    scale = _contig_out((B, H, G, D), x.dtype, dev)
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_quant_int2_grouped(
            x.data_ptr(), dt, _lib.view4(x), group_size, _lib.ptr(q8), _lib.ptr(qp), scale.data_ptr(), st
        ),
        "quant_int2",
        f"S={S} must be divisible by group_size={group_size}",
    )
    return q8, qp, scale


def quant_k_int2(k: Tensor, group_size: int = DEFAULT_INT2_GROUP_SIZE) -> tuple[Tensor, Tensor]:
    """Grouped INT2 for K (``fade/quant.py:95-112``): ``(q int8 [B,H,S,D], scale [B,H,S/G,D])``."""
    q8, _, scale = _quant_int2(k, group_size, True, False)
    return q8, scale


def quant_v_int2(v: Tensor, group_size: int = DEFAULT_INT2_GROUP_SIZE) -> tuple[Tensor, Tensor]:
    """Grouped INT2 for V (``fade/quant.py:130-150``): same arithmetic as ``quant_k_int2``."""
    q8, _, scale = _quant_int2(v, group_size, True, False)
    return q8, scale


def quant_int2_grouped_packed(x: Tensor, group_size: int) -> tuple[Tensor, Tensor]:
    """Grouped INT2 codes packed 4 per byte ``[B,H,S,D/4]`` plus scales ``[B,H,S/G,D]``.

    The codes are those of ``quant_v_int2`` (bit-exact); only the storage is
    packed, with the byte layout of ``fade/rotated_quant.py:35-48``.
    """
    _, qp, scale = _quant_int2(x, group_size, False, True)
    return qp, scale


def _dequant_call(codes: Tensor, bits: int, scale: Tensor, mode: int, group: int, dtype, shape) -> Tensor:
    dev = _lib.require_cuda(codes, scale)
    B, H, S, D = shape
    out = _contig_out((B, H, S, D), dtype, dev)
    sc = scale.to(dtype).contiguous()
    c = codes.contiguous()
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_dequant(c.data_ptr(), bits, sc.data_ptr(), mode, group, _lib.dtype_code(dtype),
                                 B, H, S, D, out.data_ptr(), st),
        "dequant",
    )
    return out


def _scale_mode(scale: Tensor, B, H, S, D) -> tuple[int, int]:
    if tuple(scale.shape) == (B, H, 1, D):
        return 0, 1
    if tuple(scale.shape) == (B, H, S, 1):
        return 1, 1
    if scale.dim() == 4 and scale.shape[:2] == (B, H) and scale.shape[3] == D and S % scale.shape[2] == 0:
        return 2, S // scale.shape[2]
    raise ValueError(f"unsupported scale shape {tuple(scale.shape)} for codes [B={B},H={H},S={S},D={D}]")


def dequant(q: Tensor, scale: Tensor, dtype: torch.dtype = torch.float16) -> Tensor:
    """``q.to(dtype) * scale.to(dtype)`` for int8 codes (``fade/quant.py:115-121``)."""
    B, H, S, D = q.shape
    mode, group = _scale_mode(scale, B, H, S, D)
    return _dequant_call(q.to(torch.int8), 8, scale, mode, group, dtype, (B, H, S, D))


def dequant_int4(packed: Tensor, scale: Tensor, dtype: torch.dtype = torch.float16) -> Tensor:
    """Unpack + dequantize INT4 (``fade/quant.py:124-127``), fused in one kernel."""
    B, H, S, Dh = packed.shape
    D = Dh * 2
    mode, group = _scale_mode(scale, B, H, S, D)
    return _dequant_call(packed, 4, scale, mode, group, dtype, (B, H, S, D))


def dequant_k_int2(q: Tensor, scale: Tensor, group_size: int = DEFAULT_INT2_GROUP_SIZE,
                   dtype: torch.dtype = torch.float16) -> Tensor:
    """``fade/quant.py:153-163``."""
    B, H, S, D = q.shape
    return _dequant_call(q.to(torch.int8), 8, scale, 2, group_size, dtype, (B, H, S, D))


def dequant_v_int2(q: Tensor, scale: Tensor, group_size: int = DEFAULT_INT2_GROUP_SIZE,
                   dtype: torch.dtype = torch.float16) -> Tensor:
    """``fade/quant.py:166-176``."""
    B, H, S, D = q.shape
    return _dequant_call(q.to(torch.int8), 8, scale, 2, group_size, dtype, (B, H, S, D))


def dequant_int2_packed(packed: Tensor, scale: Tensor, group_size: int,
                        dtype: torch.dtype = torch.float16) -> Tensor:
    """Dequantize 4-per-byte packed grouped INT2 codes."""
    B, H, S, Dq = packed.shape
    return _dequant_call(packed, 2, scale, 2, group_size, dtype, (B, H, S, Dq * 4))


def pad_to_group(x: Tensor, group_size: int) -> tuple[Tensor, int]:
    """Zero-pad the sequence dim (-2) to a multiple of ``group_size`` (``fade/quant.py:179-188``)."""
    S = x.shape[-2]
    if S % group_size == 0:
        return x, S
    total = S + group_size - (S % group_size)
    padded = torch.zeros(*x.shape[:-2], total, x.shape[-1], dtype=x.dtype, device=x.device)
    padded[..., :S, :] = x
    return padded, S


__all__ = [
    "DEFAULT_INT2_GROUP_SIZE",
    "EPS",
    "dequant",
    "dequant_int2_packed",
    "dequant_int4",
    "dequant_k_int2",
    "dequant_v_int2",
    "pad_to_group",
    "quant_int2_grouped_packed",
    "quant_k_int2",
    "quant_k_int4",
    "quant_v_int2",
    "quant_v_int4",
]
