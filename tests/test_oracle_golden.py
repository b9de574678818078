"""Pin the CPU oracle against golden vectors produced by the reference.

Bit-exact for codes, packed bytes and scales (fade/quant.py, fade/rotated_quant.py,
fade/cache.py re-RoPE); attention within the reference's own rounding.
CPU only.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import attention as oa
from oracle import quant as oq
from oracle import rope as orope
from oracle.numerics import from_bits, to_bits

DTS = ("f16", "bf16")


@pytest.mark.parametrize("dt", DTS)
def test_int4_k_v_bit_exact(dt):
    g = golden("quant")
    x = from_bits(g[f"{dt}_x"], dt)
    kp, ks = oq.quant_k_int4(x, dt)
    vp, vs = oq.quant_v_int4(x, dt)
    np.testing.assert_array_equal(kp, g[f"{dt}_k_packed"])
    np.testing.assert_array_equal(to_bits(ks, dt), g[f"{dt}_k_scale"])
    np.testing.assert_array_equal(vp, g[f"{dt}_v_packed"])
    np.testing.assert_array_equal(to_bits(vs, dt), g[f"{dt}_v_scale"])


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("G", (32, 64))
def test_int2_grouped_bit_exact(dt, G):
    g = golden("quant")
    x = from_bits(g[f"{dt}_x2"], dt)
    q, s = oq.quant_int2_grouped(x, G, dt)
    np.testing.assert_array_equal(q, g[f"{dt}_k2_g{G}_codes"])
    np.testing.assert_array_equal(to_bits(s, dt), g[f"{dt}_k2_g{G}_scale"])
    np.testing.assert_array_equal(q, g[f"{dt}_v2_g{G}_codes"])
    np.testing.assert_array_equal(to_bits(s, dt), g[f"{dt}_v2_g{G}_scale"])


def test_pack_roundtrip():
    rng = np.random.default_rng(0)
    q4 = rng.integers(-8, 8, size=(3, 5, 64)).astype(np.int8)
    np.testing.assert_array_equal(oq.unpack_int4(oq.pack_int4(q4)), q4)
    q2 = rng.integers(-2, 2, size=(3, 5, 64)).astype(np.int8)
    np.testing.assert_array_equal(oq.unpack2(oq.pack2(q2)), q2)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("D", (64, 128))
@pytest.mark.parametrize("bits", (2, 4))
def test_rotated_quant_matches_reference(dt, D, bits):
    """Scales bit-exact; codes equal except within an fp32 ulp of a rounding
    boundary (the reference's matmul sums in a different order)."""
    g = golden("rotated")
    R = g[f"R{D}"]
    x = from_bits(g[f"{dt}_D{D}_x"], dt)
    unpack = oq.unpack_int4 if bits == 4 else oq.unpack2
    for kind in ("k", "v"):
        p, s = oq.rotated_quant(x, R, bits, kind, dt)
        ref_codes = unpack(g[f"{dt}_D{D}_b{bits}_{kind}_packed"])
        codes = unpack(p)
        diff = np.abs(codes.astype(int) - ref_codes.astype(int))
        assert diff.max() <= 1
        assert (diff != 0).mean() < 2e-3
        ref_s = from_bits(g[f"{dt}_D{D}_b{bits}_{kind}_scale"], dt)
        # absmax of a rotated value: at most one fp32 ulp apart before the dtype cast
        np.testing.assert_allclose(s, ref_s, rtol=2e-2 if dt == "bf16" else 2e-3)


@pytest.mark.parametrize("dt", DTS)
def test_rerope_bit_exact(dt):
    g = golden("rope")
    k = from_bits(g[f"{dt}_k"], dt)
    out = orope.rerope_gather(k, g[f"{dt}_keep"], g[f"{dt}_cos_old"], g[f"{dt}_sin_old"],
                              g[f"{dt}_cos_new"], g[f"{dt}_sin_new"], dt)
    np.testing.assert_array_equal(to_bits(out, dt), g[f"{dt}_out"])


def _tiers_cfg1(g, dt="f16"):
    return {
        "sink_k": from_bits(g["sink_k"], dt), "sink_v": from_bits(g["sink_v"], dt),
        "recent_k": from_bits(g["recent_k"], dt), "recent_v": from_bits(g["recent_v"], dt),
        "int4_kq": g["int4_kq"], "int4_ks": from_bits(g["int4_ks"], dt),
        "int4_vq": g["int4_vq"], "int4_vs": from_bits(g["int4_vs"], dt),
    }


def test_tier_state_cfg1_matches_reference_quant():
    """The reference cache's INT4 middle equals quant_*_int4 of the middle tokens."""
    g = golden("decode_cfg1")
    k = from_bits(g["k_roped"], "f16")
    v = from_bits(g["v"], "f16")
    mid_k, mid_v = k[:, :, 4:-64], v[:, :, 4:-64]
    kp, ks = oq.quant_k_int4(mid_k, "f16")
    vp, vs = oq.quant_v_int4(mid_v, "f16")
    np.testing.assert_array_equal(kp, g["int4_kq"])
    np.testing.assert_array_equal(to_bits(ks, "f16"), g["int4_ks"])
    np.testing.assert_array_equal(vp, g["int4_vq"])
    np.testing.assert_array_equal(to_bits(vs, "f16"), g["int4_vs"])


def test_tiered_attention_cfg1_vs_reference():
    g = golden("decode_cfg1")
    q = from_bits(g["q"], "f16")
    out = oa.tiered_attention(q, _tiers_cfg1(g), "f16")
    ref = from_bits(g["out_ref"], "f16")
    ref32 = g["out_ref32"].view(np.float32)
    assert np.abs(out - ref32).max() < 1e-5
    assert np.abs(out - ref).max() < 2e-3


def test_tiered_attention_cfg3_vs_reference():
    g = golden("decode_cfg3_small")
    dt = "f16"
    q = from_bits(g["q"], dt)
    tiers = {
        "sink_k": from_bits(g["sink_k"], dt), "sink_v": from_bits(g["sink_v"], dt),
        "recent_k": from_bits(g["recent_k"], dt), "recent_v": from_bits(g["recent_v"], dt),
        "int4_kq": g["int4_kq"], "int4_ks": from_bits(g["int4_ks"], dt),
        "int4_vq2": g["int4_vq2"], "int4_vs2": from_bits(g["int4_vs2"], dt), "v_group": 64,
        "n_mid": int(g["n_mid"]),
    }
    out = oa.tiered_attention(q, tiers, dt)
    ref32 = g["out_ref32"].view(np.float32)
    assert np.abs(out - ref32).max() < 1e-5
    assert np.abs(out - from_bits(g["out_ref"], dt)).max() < 2e-3


def test_tiered_attention_rot_vs_reference():
    g = golden("decode_rot_small")
    dt = "bf16"
    q = from_bits(g["q"], dt)
    tiers = {
        "sink_k": from_bits(g["sink_k"], dt), "sink_v": from_bits(g["sink_v"], dt),
        "recent_k": from_bits(g["recent_k"], dt), "recent_v": from_bits(g["recent_v"], dt),
        "rot_kq": g["rot_kq"], "rot_ks": from_bits(g["rot_ks"], dt),
        "rot_vq": g["rot_vq"], "rot_vs": from_bits(g["rot_vs"], dt), "rot_bits": 2,
    }
    out = oa.tiered_attention(q, tiers, dt, rotation=g["R"])
    ref32 = g["out_ref32"].view(np.float32)
    # dequant rotation summed in a different order than the reference's matmul
    assert np.abs(out - ref32).max() < 1e-2
    assert np.abs(out - from_bits(g["out_ref"], dt)).max() < 1e-2
