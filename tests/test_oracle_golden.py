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
from gpu_util import assert_attn_close, dtype_ulp

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


# ----------------------------------------------------------- rotated dequant
@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("D", (64, 128))
@pytest.mark.parametrize("bits", (2, 4))
def test_rotated_dequant_matches_reference(dt, D, bits):
    """oracle.rotated_dequant on the reference's own codes and scales against
    the reference's rotated_dequant_k/_v (fade/rotated_quant.py:134-145,
    176-187): the dequant in the rotated basis is exact, the fp32 rotation
    back sums in another order than the reference's CPU matmul, so the
    dtype-rounded output is exact or one ulp off."""
    g = golden("rotated")
    R = g[f"R{D}"]
    for kind in ("k", "v"):
        packed = g[f"{dt}_D{D}_b{bits}_{kind}_packed"]
        scale = from_bits(g[f"{dt}_D{D}_b{bits}_{kind}_scale"], dt)
        out = oq.rotated_dequant(packed, scale, R, bits, dt)
        ref = from_bits(g[f"{dt}_D{D}_b{bits}_{kind}_deq"], dt).astype(np.float64)
        err = np.abs(out.astype(np.float64) - ref)
        # bound: one output ulp plus the fp32 summation error of the rotation
        # (D terms, relative 2^-24 each, of magnitude |x_rot| @ |R|)
        q = oq.unpack_int4(packed) if bits == 4 else oq.unpack2(packed)
        terms = np.abs(oq.dequant(q, scale, dt).astype(np.float64)) @ np.abs(R.astype(np.float64))
        bound = dtype_ulp(np.maximum(np.abs(ref), np.abs(out)), dt) + D * 2.0 ** -24 * terms
        assert (err <= bound).all(), (kind, (err / bound).max())
        assert (err != 0).mean() < 5e-3, (kind, (err != 0).mean())


# ------------------------------- config 3 at the benchmark configuration settings
def _gi():
    import sys

    from conftest import ROOT
    p = str(ROOT / "tests" / "golden")
    if p not in sys.path:
        sys.path.insert(0, p)
    import inputs
    return inputs


def test_cfg3_g32_inputs_and_policy_reproduce_reference():
    """The config-3 inputs regenerate bit for bit (checksums stored by the
    fixture script) and fade_b200.policy._assign_one_layer selects the same
    400 survivors as the reference's (fade/policy.py:232-274)."""
    import torch

    from fade_b200.policy import _assign_one_layer
    from fade_b200.rope import Vanilla

    gi = _gi()
    g = golden("decode_cfg3_g32")
    sc = Vanilla(theta=gi.CFG3["theta"], head_dim=gi.CFG3["D"])
    k, v, _, scores = gi.cfg3_inputs(lambda p: sc.compute_cos_sin(p, "cpu", model_dtype=torch.float16))
    assert gi.checksum(k) == int(g["k_sum"]) and gi.checksum(v) == int(g["v_sum"])
    c = gi.CFG3
    tiers = _assign_one_layer(c["S"], scores, c["n_sink"], c["recent"], c["budget"], 0)
    np.testing.assert_array_equal(tiers.numpy(), g["tiers"])
    assert int((tiers == 1).sum()) == c["budget"]


def test_oracle_cfg3_g32_vs_reference():
    """V grouped INT2 at group 32 bit-exact; attention over the reference's
    tiers within 1e-5 of its fp32 SDPA."""
    g = golden("decode_cfg3_g32")
    dt = "f16"
    v_mid = from_bits(g["v_mid"], dt)
    vq, vs = oq.quant_int2_grouped(oq.pad_to_group(v_mid, 32), 32, dt)
    np.testing.assert_array_equal(vq, g["int2_vq"])
    np.testing.assert_array_equal(to_bits(vs, dt), g["int2_vs"])
    tiers = {
        "sink_k": from_bits(g["sink_k"], dt), "sink_v": from_bits(g["sink_v"], dt),
        "recent_k": from_bits(g["recent_k"], dt), "recent_v": from_bits(g["recent_v"], dt),
        "int4_kq": g["int4_kq"], "int4_ks": from_bits(g["int4_ks"], dt),
        "int4_vq2": g["int2_vq"], "int4_vs2": from_bits(g["int2_vs"], dt), "v_group": 32,
        "n_mid": int(g["n_mid"]),
    }
    out = oa.tiered_attention(from_bits(g["q"], dt), tiers, dt)
    assert np.abs(out - g["out_ref32"].view(np.float32)).max() < 1e-5
    # the reference's own fp16 SDPA output: within 2e-3 or one fp16 ulp
    assert_attn_close(from_bits(g["out_ref"], dt), out, dt, 2e-3)


# ------------------------------------------ config 4: ragged x rotated 2-bit
def test_oracle_cfg4_ragged_rotated_vs_reference():
    """Per-sequence rotated 2-bit quantisation of the ragged config-4 batch:
    codes equal the reference's except within an fp32 ulp of a rounding
    boundary (bound measured here on ~85k vectors), scales within rounding,
    and attention over the reference's codes within bf16 tolerance of its
    fp32 SDPA."""
    gi = _gi()
    g = golden("decode_cfg4_ragged")
    c = gi.CFG4
    lens, seqs, _ = gi.cfg4_inputs()
    assert lens == g["lens"].tolist()
    R = g["R"]
    q = from_bits(g["q"], "bf16")
    ns, nr = c["n_sink"], c["recent"]
    n_diff = n_tot = 0
    for i, (k, v) in enumerate(seqs):
        assert gi.checksum(k) == int(g[f"s{i}_k_sum"]) and gi.checksum(v) == int(g[f"s{i}_v_sum"])
        kf = k.float().numpy()
        vf = v.float().numpy()
        n = kf.shape[2]
        for kind, x in (("k", kf[:, :, ns:n - nr]), ("v", vf[:, :, ns:n - nr])):
            p, s = oq.rotated_quant(x, R, 2, kind, "bf16")
            d = np.abs(oq.unpack2(p).astype(int) - oq.unpack2(g[f"s{i}_{kind}q"]).astype(int))
            assert d.max() <= 1
            n_diff += int((d != 0).sum())
            n_tot += d.size
            np.testing.assert_allclose(s, from_bits(g[f"s{i}_{kind}s"], "bf16"), rtol=2e-2)
        tiers = {"sink_k": kf[:, :, :ns], "sink_v": vf[:, :, :ns], "recent_k": kf[:, :, n - nr:],
                 "recent_v": vf[:, :, n - nr:], "rot_kq": g[f"s{i}_kq"], "rot_ks": from_bits(g[f"s{i}_ks"], "bf16"),
                 "rot_vq": g[f"s{i}_vq"], "rot_vs": from_bits(g[f"s{i}_vs"], "bf16"), "rot_bits": 2}
        out = oa.tiered_attention(q[i:i + 1], tiers, "bf16", rotation=R)
        assert np.abs(out - g[f"s{i}_out_ref32"].view(np.float32)).max() < 1e-2
    assert n_diff / n_tot < 2e-3, n_diff / n_tot
