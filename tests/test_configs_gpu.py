"""Benchmark configurations 3 and 4 on the GPU against fixtures made by running the
reference (tests/golden/make_golden.py).  The inputs are regenerated here from
their seeds (tests/golden/inputs.py) and checked against the fixture's
checksums first, so the GPU sees exactly the bits the reference saw."""

from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, golden
from gpu_util import assert_attn_close, t_bits, t_from_bits, t_vals
from oracle import attention as oa
from oracle import quant as oq
from oracle.numerics import from_bits, to_bits
from test_cache_gpu import _oracle_survivors

sys.path.insert(0, str(ROOT / "tests" / "golden"))
import inputs as gi  # noqa: E402

pytestmark = pytest.mark.gpu


def test_cfg3_g32_h2o_eviction_and_decode(cuda_device):
    """Mistral-7B shape, H2O: 4096-token prompt, Dirichlet(0.1) scores summed
    over heads, 400 INT4 survivors (policy on the GPU), eviction re-RoPE, K INT4
    + V grouped INT2 at group 32, fused decode over the compacted cache."""
    from fade_b200.cache import TieredKVCache
    from fade_b200.policy import _assign_one_layer
    from fade_b200.rope import Vanilla

    g = golden("decode_cfg3_g32")
    c = gi.CFG3
    scheme = Vanilla(theta=c["theta"], head_dim=c["D"])
    k, v, q, scores = gi.cfg3_inputs(lambda p: scheme.compute_cos_sin(p, "cpu", model_dtype=torch.float16))
    assert gi.checksum(k) == int(g["k_sum"]) and gi.checksum(v) == int(g["v_sum"])
    dev = cuda_device
    k, v, q, scores = k.to(dev), v.to(dev), q.to(dev), scores.to(dev)
    cache = TieredKVCache(n_sink=c["n_sink"], recent_window=c["recent"], int4_budget=c["budget"],
                          dtype=torch.float16, rope_theta=c["theta"], head_dim=c["D"], middle_v_bits=2,
                          rope_scheme=scheme, v_int2_group_size=c["group"])
    cache.update(k, v, 0)
    tiers = _assign_one_layer(c["S"], scores, c["n_sink"], c["recent"], c["budget"], 0)
    np.testing.assert_array_equal(tiers.cpu().numpy(), g["tiers"])
    cache.apply_tier_assignment(0, tiers)
    st = cache._layers[0]
    # V: grouped INT2 codes and scales bit-exact with the reference's quant_v_int2(group 32)
    np.testing.assert_array_equal(st.int4_vq.cpu().numpy(), g["int2_vq"])
    np.testing.assert_array_equal(t_bits(st.int4_vs), g["int2_vs"])
    np.testing.assert_array_equal(t_bits(st.sink_v), g["sink_v"])
    np.testing.assert_array_equal(t_bits(st.fp16_v), g["recent_v"])
    # K: bit-exact with the reference's arithmetic on this device's cos/sin
    kk, kt = _oracle_survivors(cache, t_bits(k), g["tiers"], "f16", k.device)
    fp = kk[:, :, kt == 0]
    np.testing.assert_array_equal(t_bits(st.sink_k), to_bits(fp[:, :, :4], "f16"))
    np.testing.assert_array_equal(t_bits(st.fp16_k), to_bits(fp[:, :, 4:], "f16"))
    kq, ks = oq.quant_k_int4(kk[:, :, kt == 1], "f16")
    np.testing.assert_array_equal(st.int4_kq.cpu().numpy(), kq)
    np.testing.assert_array_equal(t_bits(st.int4_ks), to_bits(ks, "f16"))
    # fused decode over the compacted cache vs the reference's fp32 SDPA
    out = t_vals(cache.decode_attention(0, q))
    assert_attn_close(out, t_vals(t_from_bits(g["out_ref32"], "f32")), "f16", 2e-3)


def test_cfg3_reassignment_without_host_sync(cuda_device):
    """The config-3 reassignment with the tier counts known on the host
    (``assign_counts`` from the budgets): ``_assign_one_layer`` on the GPU
    scores and ``apply_tier_assignment(..., counts=...)`` make no host
    synchronisation (torch's sync debug mode raises on one), and every tier
    of the cache equals the mask path's bit for bit."""
    from fade_b200.cache import TieredKVCache
    from fade_b200.policy import _assign_one_layer, assign_counts
    from fade_b200.rope import Vanilla

    c = gi.CFG3
    scheme = Vanilla(theta=c["theta"], head_dim=c["D"])
    k, v, q, scores = gi.cfg3_inputs(lambda p: scheme.compute_cos_sin(p, "cpu", model_dtype=torch.float16))
    dev = cuda_device
    k, v, q, scores = k.to(dev), v.to(dev), q.to(dev), scores.to(dev)
    caches = []
    for _ in range(2):
        cache = TieredKVCache(n_sink=c["n_sink"], recent_window=c["recent"], int4_budget=c["budget"],
                              dtype=torch.float16, rope_theta=c["theta"], head_dim=c["D"], middle_v_bits=2,
                              rope_scheme=scheme, v_int2_group_size=c["group"])
        cache.update(k, v, 0)
        caches.append(cache)
    args = (c["S"], c["n_sink"], c["recent"], c["budget"], 0)
    caches[0].apply_tier_assignment(0, _assign_one_layer(args[0], scores, *args[1:]))
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        tiers = _assign_one_layer(args[0], scores, *args[1:])
        caches[1].apply_tier_assignment(0, tiers, counts=assign_counts(*args))
    finally:
        torch.cuda.set_sync_debug_mode(0)
    a, b = caches[0]._layers[0], caches[1]._layers[0]
    assert a.next_position == b.next_position
    for name in ("sink_k", "sink_v", "sink_pos", "fp16_k", "fp16_v", "fp16_pos", "int4_kq", "int4_ks",
                 "int4_vq", "int4_vs", "int4_pos"):
        ta, tb = getattr(a, name), getattr(b, name)
        assert (ta is None) == (tb is None), name
        if ta is not None:
            assert ta.shape == tb.shape and torch.equal(ta, tb), name
    assert torch.equal(caches[0].decode_attention(0, q), caches[1].decode_attention(0, q))


def test_cfg4_ragged_rotated_decode(cuda_device):
    """Qwen2.5-7B shape, ragged batch (per-sequence middle lengths, ragged
    unit grid) with the rotated 2-bit middle: GPU quantiser codes against the
    reference's, then one fused decode call over all sequences against the
    reference's per-sequence dequant + SDPA."""
    from fade_b200.attention import FPTier, RotTier, tiered_decode_attention
    from fade_b200.rotated_quant import rotated_quant_k, rotated_quant_v

    g = golden("decode_cfg4_ragged")
    c = gi.CFG4
    lens, seqs, q = gi.cfg4_inputs()
    assert lens == g["lens"].tolist()
    dev = cuda_device
    R = torch.from_numpy(g["R"]).to(dev)
    ns, nr, D, H = c["n_sink"], c["recent"], c["D"], c["Hkv"]
    nseq = len(lens)
    mids = [n - ns - nr for n in lens]
    cap = -(-max(mids) // 128) * 128
    kp = torch.zeros(nseq, H, cap, D // 4, dtype=torch.uint8, device=dev)
    vp = torch.zeros_like(kp)
    ks = torch.zeros(nseq, H, 1, D, dtype=torch.bfloat16, device=dev)
    vs = torch.zeros(nseq, H, cap, 1, dtype=torch.bfloat16, device=dev)
    sink_k = torch.empty(nseq, H, ns, D, dtype=torch.bfloat16, device=dev)
    sink_v = torch.empty_like(sink_k)
    rec_k = torch.empty(nseq, H, nr, D, dtype=torch.bfloat16, device=dev)
    rec_v = torch.empty_like(rec_k)
    n_diff = n_tot = 0
    for i, (k, v) in enumerate(seqs):
        assert gi.checksum(k) == int(g[f"s{i}_k_sum"]) and gi.checksum(v) == int(g[f"s{i}_v_sum"])
        k, v = k.to(dev), v.to(dev)
        n = k.shape[2]
        for kind, fn, x in (("k", rotated_quant_k, k[:, :, ns:n - nr]), ("v", rotated_quant_v, v[:, :, ns:n - nr])):
            p, s = fn(x.contiguous(), R, bits=2)
            d = np.abs(oq.unpack2(p.cpu().numpy()).astype(int) - oq.unpack2(g[f"s{i}_{kind}q"]).astype(int))
            assert d.max() <= 1
            n_diff += int((d != 0).sum())
            n_tot += d.size
        m = mids[i]
        # the decode reads the reference's own codes and scales
        kp[i, :, :m] = torch.from_numpy(g[f"s{i}_kq"][0]).to(dev)
        vp[i, :, :m] = torch.from_numpy(g[f"s{i}_vq"][0]).to(dev)
        ks[i] = t_from_bits(g[f"s{i}_ks"][0], "bf16", dev)
        vs[i, :, :m] = t_from_bits(g[f"s{i}_vs"][0], "bf16", dev)
        sink_k[i], sink_v[i] = k[0, :, :ns], v[0, :, :ns]
        rec_k[i], rec_v[i] = k[0, :, n - nr:], v[0, :, n - nr:]
    assert n_diff / n_tot < 2e-3
    lens_t = torch.tensor(mids, dtype=torch.int32, device=dev)
    units = np.repeat([-(-m // 128) for m in mids], H)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(units)]).astype(np.int32)).to(dev)
    mid = RotTier(kp, ks, vp, vs, bits=2, rotation=R, lens=lens_t, max_len=cap)
    qd = q.to(dev)
    out = t_vals(tiered_decode_attention(qd, [FPTier(sink_k, sink_v), mid, FPTier(rec_k, rec_v)], cu_units=cu))
    # The reference rounds the un-rotated K/V to bf16 (rnd(rnd(q*s) @ R),
    # fade/rotated_quant.py:134-145); the fused kernel attends in the rotated
    # basis and has no such intermediate.  So: strict tolerance against the
    # exact math on the same codes, and against the reference's output the
    # tolerance plus the reference's own distance from that exact math.
    for i, (k, v) in enumerate(seqs):
        n = k.shape[2]
        kf, vf = k.float().numpy(), v.float().numpy()
        tiers = {"sink_k": kf[:, :, :ns], "sink_v": vf[:, :, :ns], "recent_k": kf[:, :, n - nr:],
                 "recent_v": vf[:, :, n - nr:], "rot_kq": g[f"s{i}_kq"], "rot_ks": from_bits(g[f"s{i}_ks"], "bf16"),
                 "rot_vq": g[f"s{i}_vq"], "rot_vs": from_bits(g[f"s{i}_vs"], "bf16"), "rot_bits": 2,
                 "rot_exact": True}
        exact = oa.tiered_attention(q[i:i + 1].float().numpy(), tiers, "bf16", rotation=g["R"])
        assert_attn_close(out[i:i + 1], exact, "bf16", 1e-2)
        ref = t_vals(t_from_bits(g[f"s{i}_out_ref32"], "f32")).astype(np.float64)
        ref_dev = np.abs(ref - exact)
        lim = 1e-2 + ref_dev
        err = np.abs(out[i:i + 1] - ref)
        print(f"[cfg4 seq {i}] max|out-ref| {err.max():.3e}, reference's own max|ref-exact| {ref_dev.max():.3e}")
        assert (err <= np.maximum(lim, 1e-2 + 2 * np.abs(ref) * 2.0 ** -8)).all()
