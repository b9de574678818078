"""Tiered decode attention oracle -- TEST INFRASTRUCTURE ONLY.

Restates the reference's decode step: TieredKVCache._materialize
(fade/cache.py:693-808: cat(sink, dequant(middle), recent), every dequant
rounded to the model dtype) followed by scaled-dot-product attention with GQA
(transformers sdpa_attention.py:40-62: kv head h serves query heads
h*g .. h*g+g-1).  The attention itself is evaluated in float64, so the oracle
is the exact value of the reference's math on the dequantised tiers; the
reference's own fp16/bf16 SDPA differs from it by its output rounding, which
the tolerances (2e-3 fp16, 1e-2 bf16) cover.
"""

from __future__ import annotations

import numpy as np

from oracle import quant as oq


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None) -> np.ndarray:
    """q [B,Hq,Sq,D], k/v [B,Hkv,S,D] (float) -> [B,Hq,Sq,D] float64, non-causal."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, Hq, Sq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    kk = np.repeat(k, g, axis=1)
    vv = np.repeat(v, g, axis=1)
    s = np.einsum("bhqd,bhsd->bhqs", q, kk) * scale
    if s.shape[-1] == 0:
        return np.zeros(q.shape)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqs,bhsd->bhqd", p, vv)


def materialize(tiers: dict, dt: str, rotation: np.ndarray | None = None):
    """Build dequantised K/V from a tier dict (any subset of keys):
      sink_k/sink_v [B,H,n,D]; recent_k/recent_v [B,H,r,D] (dtype values)
      int4_kq/int4_ks/int4_vq/int4_vs  (INT4 K per-channel, INT4 V per-token)
      int4_vq2/int4_vs2/v_group        (V grouped INT2 instead of INT4 V, codes int8 [B,H,S_pad,D])
      n_mid                            (valid middle tokens; padding trimmed)
      rot_kq/rot_ks/rot_vq/rot_vs/rot_bits  (rotated middle; rot_exact=True skips the
                                             reference's rounding of the un-rotated K/V)
    Order of the concatenation does not change attention; the reference's is kept."""
    parts_k, parts_v = [], []
    if "sink_k" in tiers:
        parts_k.append(tiers["sink_k"])
        parts_v.append(tiers["sink_v"])
    if "int4_kq" in tiers:
        n = tiers.get("n_mid", tiers["int4_kq"].shape[2])
        k4 = oq.dequant_int4(tiers["int4_kq"], tiers["int4_ks"], dt)[..., :n, :]
        if "int4_vq2" in tiers:
            v4 = oq.dequant_grouped(tiers["int4_vq2"], tiers["int4_vs2"], tiers["v_group"], dt)[..., :n, :]
        else:
            v4 = oq.dequant_int4(tiers["int4_vq"], tiers["int4_vs"], dt)[..., :n, :]
        parts_k.append(k4)
        parts_v.append(v4)
    if "rot_kq" in tiers:
        bits = int(tiers["rot_bits"])
        if tiers.get("rot_exact"):
            # diagnostic form: rnd(code * scale) @ R in float64, without the
            # reference's final rounding of the un-rotated K/V to the dtype
            unpack = oq.unpack_int4 if bits == 4 else oq.unpack2
            Rd = np.asarray(rotation, dtype=np.float64)
            for key_q, key_s, parts in (("rot_kq", "rot_ks", parts_k), ("rot_vq", "rot_vs", parts_v)):
                parts.append(oq.dequant(unpack(tiers[key_q]), tiers[key_s], dt).astype(np.float64) @ Rd)
        else:
            parts_k.append(oq.rotated_dequant(tiers["rot_kq"], tiers["rot_ks"], rotation, bits, dt))
            parts_v.append(oq.rotated_dequant(tiers["rot_vq"], tiers["rot_vs"], rotation, bits, dt))
    if "recent_k" in tiers:
        parts_k.append(tiers["recent_k"])
        parts_v.append(tiers["recent_v"])
    return np.concatenate(parts_k, axis=2), np.concatenate(parts_v, axis=2)


def tiered_attention(q: np.ndarray, tiers: dict, dt: str, rotation=None, scale=None) -> np.ndarray:
    k, v = materialize(tiers, dt, rotation)
    return sdpa(q, k, v, scale)
