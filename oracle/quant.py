"""Numpy restatement of the reference's quantisers -- TEST INFRASTRUCTURE ONLY.

Inputs are float32 arrays holding values representable in `dt` ("f16",
"bf16" or "f32"); outputs are bit-exact with the reference:
  quant_k_int4 / quant_v_int4      fade/quant.py:61-92
  _pack_int4 / _unpack_int4        fade/quant.py:26-58
  quant_int2_grouped               fade/quant.py:95-112, 130-150
  dequant                          fade/quant.py:115-176
  pack2 / unpack2                  fade/rotated_quant.py:35-69
  rotated_quant / rotated_dequant  fade/rotated_quant.py:106-187 (see note)
  age_out_int4                     extension (no reference counterpart)

Rotation note: the reference computes ``x @ R.T`` with torch's CPU matmul;
this restatement (and the CUDA kernel) accumulate the D products
sequentially in fp32 with separate roundings, so codes can differ from the
reference's where a rotated value lies within an ulp of a rounding boundary.
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import eps, rnd


def _recip_times(absmax: np.ndarray, qmax: float, dt: str) -> np.ndarray:
    """torch's ``qmax / absmax`` = rnd(rnd(1/absmax) * qmax)  (Tensor.__rtruediv__)."""
    with np.errstate(divide="ignore"):
        r = rnd(np.float32(1.0) / absmax.astype(np.float32), dt)
    return rnd(r * np.float32(qmax), dt)


def _codes(x: np.ndarray, inv: np.ndarray, lo: int, hi: int, dt: str) -> np.ndarray:
    with np.errstate(invalid="ignore", over="ignore"):
        y = rnd(x * inv, dt)
        y = np.rint(y)  # half to even, like torch.round
        y = np.clip(y, lo, hi)
    y = np.where(np.isnan(y), 0.0, y)  # 0 * inf -> NaN -> int8 0 (torch on CPU)
    return y.astype(np.int8)


def pack_int4(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q).astype(np.int16) & 0xF
    return ((q[..., 0::2] << 4) | q[..., 1::2]).astype(np.uint8)


def unpack_int4(p: np.ndarray) -> np.ndarray:
    p = np.asarray(p).astype(np.int16)
    hi = (p >> 4) & 0xF
    lo = p & 0xF
    hi = hi - ((hi & 8) << 1)
    lo = lo - ((lo & 8) << 1)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = hi
    out[..., 1::2] = lo
    return out


def pack2(q: np.ndarray) -> np.ndarray:
    q = (np.asarray(q).astype(np.int16) & 3).astype(np.uint8)
    return ((q[..., 0::4] << 6) | (q[..., 1::4] << 4) | (q[..., 2::4] << 2) | q[..., 3::4]).astype(np.uint8)


def unpack2(p: np.ndarray) -> np.ndarray:
    p = np.asarray(p).astype(np.int16)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 4,), dtype=np.int8)
    for j in range(4):
        f = (p >> (6 - 2 * j)) & 3
        out[..., j::4] = f - ((f & 2) << 1)
    return out


def quant_k_int4(k: np.ndarray, dt: str):
    """-> (packed uint8 [...,S,D/2], scale float32 [...,1,D])."""
    k = np.asarray(k, dtype=np.float32)
    absmax = np.maximum(np.abs(k).max(axis=-2, keepdims=True), eps(dt))
    inv = _recip_times(absmax, 7.0, dt)
    scale = rnd(absmax / np.float32(7.0), dt)
    return pack_int4(_codes(k, inv, -8, 7, dt)), scale


def quant_v_int4(v: np.ndarray, dt: str):
    """-> (packed uint8 [...,S,D/2], scale float32 [...,S,1])."""
    v = np.asarray(v, dtype=np.float32)
    absmax = np.maximum(np.abs(v).max(axis=-1, keepdims=True), eps(dt))
    inv = _recip_times(absmax, 7.0, dt)
    scale = rnd(absmax / np.float32(7.0), dt)
    return pack_int4(_codes(v, inv, -8, 7, dt)), scale


def quant_int2_grouped(x: np.ndarray, group: int, dt: str):
    """-> (codes int8 [B,H,S,D], scale float32 [B,H,S/G,D])."""
    x = np.asarray(x, dtype=np.float32)
    B, H, S, D = x.shape
    if S % group:
        raise ValueError(f"S={S} must be divisible by group_size={group}")
    xg = x.reshape(B, H, S // group, group, D)
    absmax = np.maximum(np.abs(xg).max(axis=-2, keepdims=True), eps(dt))
    inv = _recip_times(absmax, 1.0, dt)
    scale = rnd(absmax / np.float32(1.0), dt)
    q = _codes(xg, inv, -2, 1, dt)
    return q.reshape(B, H, S, D), scale[..., 0, :]


def dequant(q: np.ndarray, scale: np.ndarray, dt: str) -> np.ndarray:
    """rnd(fp(q) * fp(scale)) with numpy broadcasting."""
    return rnd(np.asarray(q, dtype=np.float32) * np.asarray(scale, dtype=np.float32), dt)


def dequant_int4(packed: np.ndarray, scale: np.ndarray, dt: str) -> np.ndarray:
    return dequant(unpack_int4(packed), scale, dt)


def dequant_grouped(q: np.ndarray, scale: np.ndarray, group: int, dt: str) -> np.ndarray:
    B, H, S, D = q.shape
    full = np.repeat(scale, group, axis=2)
    return dequant(q, full, dt)


def pad_to_group(x: np.ndarray, group: int) -> np.ndarray:
    S = x.shape[-2]
    if S % group == 0:
        return x
    total = S + group - S % group
    out = np.zeros(x.shape[:-2] + (total, x.shape[-1]), dtype=x.dtype)
    out[..., :S, :] = x
    return out


_BITS = {4: (-8, 7), 3: (-4, 3), 2: (-2, 1)}


def rotate(x: np.ndarray, R: np.ndarray) -> np.ndarray:
    """x @ R^T in fp32, products and sums rounded separately, e = 0..D-1 in order."""
    x = np.asarray(x, dtype=np.float32)
    R = np.asarray(R, dtype=np.float32)
    acc = np.zeros(x.shape, dtype=np.float32)
    for e in range(x.shape[-1]):
        acc = (acc + (x[..., e : e + 1] * R[:, e]).astype(np.float32)).astype(np.float32)
    return acc


def rotate_back(xr: np.ndarray, R: np.ndarray) -> np.ndarray:
    """xr @ R in fp32 with the same sequential accumulation."""
    xr = np.asarray(xr, dtype=np.float32)
    R = np.asarray(R, dtype=np.float32)
    acc = np.zeros(xr.shape, dtype=np.float32)
    for e in range(xr.shape[-1]):
        acc = (acc + (xr[..., e : e + 1] * R[e, :]).astype(np.float32)).astype(np.float32)
    return acc


def rotated_quant(x: np.ndarray, R: np.ndarray, bits: int, kind: str, dt: str):
    """kind 'k': per-channel scale [...,1,D]; 'v': per-token [...,S,1].  Math in fp32."""
    lo, hi = _BITS[bits]
    xr = rotate(x, R)
    axis = -2 if kind == "k" else -1
    absmax = np.maximum(np.abs(xr).max(axis=axis, keepdims=True), np.float32(1e-8))
    inv = _recip_times(absmax, float(hi), "f32")
    scale = rnd(absmax / np.float32(hi), dt)
    q = _codes(xr, inv, lo, hi, "f32")
    if bits == 4:
        return pack_int4(q), scale
    if bits == 2:
        return pack2(q), scale
    return q, scale


def rotated_dequant(packed: np.ndarray, scale: np.ndarray, R: np.ndarray, bits: int, dt: str) -> np.ndarray:
    if bits == 4:
        q = unpack_int4(packed)
    elif bits == 2:
        q = unpack2(packed)
    else:
        q = np.asarray(packed, dtype=np.int8)
    xr = dequant(q, scale, dt)
    return rnd(rotate_back(xr, R), dt)


def age_out_int4(k_tok: np.ndarray, v_tok: np.ndarray, k_scale: np.ndarray, dt: str):
    """One token per (b,h): K codes against a frozen per-channel scale
    (clamp(rint(x / s)), 0 where s == 0), V as quant_v_int4.
    k_tok, v_tok: [B,H,D]; k_scale: [B,H,D].  -> (k_packed [B,H,D/2], v_packed, v_scale [B,H])."""
    k_tok = np.asarray(k_tok, dtype=np.float32)
    s = np.asarray(k_scale, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.clip(np.rint(k_tok / s), -8, 7)
    y = np.where(s > 0, y, 0.0)
    y = np.where(np.isnan(y), 0.0, y).astype(np.int8)
    vp, vs = quant_v_int4(v_tok[..., None, :], dt)
    return pack_int4(y), vp[..., 0, :], vs[..., 0, 0]
