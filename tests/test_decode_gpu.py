"""K2 fused tiered decode attention on the GPU vs the reference's golden outputs
and the CPU oracle.  Tolerances (max-abs): 2e-3 fp16, 1e-2 bf16."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import assert_attn_close, np_to_dt_tensor, seeded_outliers, t_bits, t_from_bits, t_vals
from oracle import attention as oa
from oracle import quant as oq
from oracle.numerics import from_bits, to_bits

pytestmark = pytest.mark.gpu
TOL = {"f16": 2e-3, "bf16": 1e-2}   # north-star max-abs tolerances (see assert_attn_close)


def _fp(g, name, dt):
    return t_from_bits(g[name], dt)


def test_cfg1_golden(cuda_device):
    """Qwen2.5-0.5B shape (config 1) through the reference cache's own tiers."""
    from fade_b200.attention import FPTier, Int4Tier, tiered_decode_attention

    g = golden("decode_cfg1")
    dt = "f16"
    q = _fp(g, "q", dt)
    tiers = [
        FPTier(_fp(g, "sink_k", dt), _fp(g, "sink_v", dt)),
        Int4Tier(torch.from_numpy(g["int4_kq"]).cuda(), _fp(g, "int4_ks", dt),
                 torch.from_numpy(g["int4_vq"]).cuda(), _fp(g, "int4_vs", dt)),
        FPTier(_fp(g, "recent_k", dt), _fp(g, "recent_v", dt)),
    ]
    out = t_vals(tiered_decode_attention(q, tiers))
    ref = from_bits(g["out_ref"], dt)
    ref32 = g["out_ref32"].view(np.float32)
    assert_attn_close(out, ref, dt, TOL[dt])
    assert_attn_close(out, ref32, dt, TOL[dt])


def test_cfg3_small_golden(cuda_device):
    """K INT4 + V grouped INT2 (G=64, the reference's default) after H2O eviction."""
    from fade_b200.attention import FPTier, Int4K2VTier, tiered_decode_attention

    g = golden("decode_cfg3_small")
    dt = "f16"
    n_mid = int(g["n_mid"])
    kq = g["int4_kq"]                       # [B,H,n_mid,D/2]
    vq8 = g["int4_vq2"]                     # int8 [B,H,S_pad,D]
    S_pad = vq8.shape[2]
    kq_pad = np.zeros(kq.shape[:2] + (S_pad, kq.shape[3]), dtype=np.uint8)
    kq_pad[:, :, :n_mid] = kq
    q = _fp(g, "q", dt)
    tiers = [
        FPTier(_fp(g, "sink_k", dt), _fp(g, "sink_v", dt)),
        Int4K2VTier(torch.from_numpy(kq_pad).cuda(), _fp(g, "int4_ks", dt),
                    torch.from_numpy(oq.pack2(vq8)).cuda(), _fp(g, "int4_vs2", dt), group=64, length=n_mid),
        FPTier(_fp(g, "recent_k", dt), _fp(g, "recent_v", dt)),
    ]
    out = t_vals(tiered_decode_attention(q, tiers))
    assert_attn_close(out, from_bits(g["out_ref"], dt), dt, TOL[dt])
    assert_attn_close(out, g["out_ref32"].view(np.float32), dt, TOL[dt])


def test_rot2_golden(cuda_device):
    """Rotated 2-bit backend (config 4 shape), bf16."""
    from fade_b200.attention import FPTier, RotTier, tiered_decode_attention

    g = golden("decode_rot_small")
    dt = "bf16"
    q = _fp(g, "q", dt)
    R = torch.from_numpy(g["R"]).cuda()
    tiers = [
        FPTier(_fp(g, "sink_k", dt), _fp(g, "sink_v", dt)),
        RotTier(torch.from_numpy(g["rot_kq"]).cuda(), _fp(g, "rot_ks", dt),
                torch.from_numpy(g["rot_vq"]).cuda(), _fp(g, "rot_vs", dt), bits=2, rotation=R),
        FPTier(_fp(g, "recent_k", dt), _fp(g, "recent_v", dt)),
    ]
    out = t_vals(tiered_decode_attention(q, tiers))
    # The reference dequantises in the rotated basis, rotates back in fp32 and
    # rounds the un-rotated K/V to bf16 (fade/rotated_quant.py:134-187); the
    # fused kernel works in the rotated basis (q_rot = q R^T, out = o_rot R), so
    # that last per-element rounding cannot be reproduced: allow atol + 2 output
    # ulps (exact rotated-basis math already sits at ~0.6 of this bound).
    assert_attn_close(out, from_bits(g["out_ref"], dt), dt, TOL[dt], ulps=2, additive=True)
    assert_attn_close(out, g["out_ref32"].view(np.float32), dt, TOL[dt], ulps=2, additive=True)


def _random_int4_case(B, Hq, Hkv, D, n_sink, n_mid, n_rec, dt, seed, n_q=1):
    x = seeded_outliers((B, Hkv, n_sink + n_mid + n_rec, D), seed, dt)
    v = seeded_outliers((B, Hkv, n_sink + n_mid + n_rec, D), seed + 1, dt)
    rng = np.random.default_rng(seed + 2)
    q = from_bits_dt(rng.standard_normal((B, Hq, n_q, D)).astype(np.float32), dt)
    mk, mv = x[:, :, n_sink:n_sink + n_mid], v[:, :, n_sink:n_sink + n_mid]
    if n_mid:
        kp, ks = oq.quant_k_int4(mk, dt)
        vp, vs = oq.quant_v_int4(mv, dt)
    else:
        kp = vp = np.zeros((B, Hkv, 0, D // 2), np.uint8)
        ks, vs = np.zeros((B, Hkv, 1, D), np.float32), np.zeros((B, Hkv, 0, 1), np.float32)
    tiers = {"sink_k": x[:, :, :n_sink], "sink_v": v[:, :, :n_sink],
             "int4_kq": kp, "int4_ks": ks, "int4_vq": vp, "int4_vs": vs,
             "recent_k": x[:, :, n_sink + n_mid:], "recent_v": v[:, :, n_sink + n_mid:]}
    return q, tiers


def from_bits_dt(x, dt):
    from oracle.numerics import rnd

    return rnd(x, dt)


def _torch_tiers(tiers, dt):
    from fade_b200.attention import FPTier, Int4Tier

    out = []
    if tiers["sink_k"].shape[2]:
        out.append(FPTier(np_to_dt_tensor(tiers["sink_k"], dt), np_to_dt_tensor(tiers["sink_v"], dt)))
    if tiers["int4_kq"].shape[2]:
        out.append(Int4Tier(torch.from_numpy(tiers["int4_kq"]).cuda(), np_to_dt_tensor(tiers["int4_ks"], dt),
                            torch.from_numpy(tiers["int4_vq"]).cuda(), np_to_dt_tensor(tiers["int4_vs"], dt)))
    if tiers["recent_k"].shape[2]:
        out.append(FPTier(np_to_dt_tensor(tiers["recent_k"], dt), np_to_dt_tensor(tiers["recent_v"], dt)))
    return out


@pytest.mark.parametrize(
    "B,Hq,Hkv,D,n_sink,n_mid,n_rec,dt,n_q",
    [
        (2, 32, 8, 128, 4, 1000, 64, "bf16", 1),     # Llama-8B head shape
        (1, 14, 2, 64, 4, 1980, 64, "f16", 1),       # config 1
        (3, 8, 8, 128, 4, 129, 5, "f16", 1),         # MHA (g=1), ragged edge of a unit
        (1, 16, 1, 64, 0, 300, 0, "bf16", 1),        # g=16 (two n-tiles), no FP tiers
        (2, 28, 4, 128, 4, 1, 64, "bf16", 1),        # a single middle token, g=7
        (1, 8, 2, 128, 4, 0, 64, "f16", 1),          # empty middle
        (2, 8, 2, 64, 4, 777, 64, "f16", 3),         # several query positions (rows = 12)
        (1, 64, 8, 128, 4, 4096, 128, "bf16", 1),    # Llama-70B head shape
    ],
)
def test_random_vs_oracle(cuda_device, B, Hq, Hkv, D, n_sink, n_mid, n_rec, dt, n_q):
    from fade_b200.attention import tiered_decode_attention

    q, tiers = _random_int4_case(B, Hq, Hkv, D, n_sink, n_mid, n_rec, dt, seed=B * 1000 + n_mid, n_q=n_q)
    ref = oa.tiered_attention(q, tiers, dt)
    out = t_vals(tiered_decode_attention(np_to_dt_tensor(q, dt), _torch_tiers(tiers, dt)))
    assert_attn_close(out, ref, dt, TOL[dt])


def test_forced_cta_counts_agree(cuda_device):
    """The split-K partition (persistent CTA count) must not change results beyond rounding."""
    from fade_b200.attention import tiered_decode_attention

    q, tiers = _random_int4_case(2, 32, 8, 128, 4, 3000, 64, "bf16", seed=5)
    qt = np_to_dt_tensor(q, "bf16")
    tt = _torch_tiers(tiers, "bf16")
    ref = oa.tiered_attention(q, tiers, "bf16")
    for n in (1, 7, 64, 300, 2000):
        out = t_vals(tiered_decode_attention(qt, tt, n_ctas=n))
        assert_attn_close(out, ref, "bf16", TOL["bf16"])


def test_device_lengths_and_ragged(cuda_device):
    """Per-row lengths from device memory, uniform grid (capacity) and ragged cu_units."""
    from fade_b200.attention import FPTier, Int4Tier, tiered_decode_attention

    dt = "bf16"
    B, Hq, Hkv, D, cap = 3, 8, 2, 128, 1024
    lens = np.array([1000, 17, 640], dtype=np.int32)
    x = seeded_outliers((B, Hkv, cap, D), 21, dt)
    v = seeded_outliers((B, Hkv, cap, D), 22, dt)
    kp = np.zeros((B, Hkv, cap, D // 2), np.uint8)
    vp = np.zeros_like(kp)
    ks = np.zeros((B, Hkv, 1, D), np.float32)
    vs = np.full((B, Hkv, cap, 1), np.nan, np.float32)   # garbage past each length must not leak
    for b in range(B):
        n = lens[b]
        kp[b:b + 1, :, :n], ks[b:b + 1] = oq.quant_k_int4(x[b:b + 1, :, :n], dt)
        vp[b:b + 1, :, :n], vs[b:b + 1, :, :n] = oq.quant_v_int4(v[b:b + 1, :, :n], dt)
    rng = np.random.default_rng(0)
    q = from_bits_dt(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    sink = seeded_outliers((B, Hkv, 4, D), 23, dt)
    qt = np_to_dt_tensor(q, dt)
    lens_t = torch.from_numpy(lens).cuda()
    mid = Int4Tier(torch.from_numpy(kp).cuda(), np_to_dt_tensor(ks, dt), torch.from_numpy(vp).cuda(),
                   np_to_dt_tensor(np.nan_to_num(vs), dt), lens=lens_t, max_len=cap)
    # NaN scales beyond the length: write them through bits
    vs_t = mid.v_scale
    for b in range(B):
        vs_t[b, :, lens[b]:] = float("nan")
    fp = FPTier(np_to_dt_tensor(sink, dt), np_to_dt_tensor(sink, dt))
    units = np.repeat(-(-lens // 128), Hkv)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(units)]).astype(np.int32)).cuda()
    for use_cu in (False, True):
        out = t_vals(tiered_decode_attention(qt, [fp, mid], cu_units=cu if use_cu else None))
        for b in range(B):
            n = lens[b]
            t = {"sink_k": sink[b:b + 1], "sink_v": sink[b:b + 1], "int4_kq": kp[b:b + 1, :, :n],
                 "int4_ks": ks[b:b + 1], "int4_vq": vp[b:b + 1, :, :n], "int4_vs": vs[b:b + 1, :, :n]}
            ref = oa.tiered_attention(q[b:b + 1], t, dt)
            assert_attn_close(out[b:b + 1], ref, dt, TOL[dt])


def test_repeat_calls_are_stable(cuda_device):
    from fade_b200.attention import tiered_decode_attention

    q, tiers = _random_int4_case(4, 32, 8, 128, 4, 2000, 64, "bf16", seed=9)
    qt = np_to_dt_tensor(q, "bf16")
    tt = _torch_tiers(tiers, "bf16")
    a = tiered_decode_attention(qt, tt).clone()
    for _ in range(5):
        b = tiered_decode_attention(qt, tt)
        assert torch.equal(a, b)


@pytest.mark.parametrize("fused,S,cap,L", [(True, 600, 600, 2), (False, 600, 600, 2), (True, 194, 128, 2),
                                           (False, 194, 128, 2), (True, 194, 300, 1), (False, 194, 300, 1)])
def test_decoder_step_matches_oracle(cuda_device, fused, S, cap, L):
    """Multi-layer TieredDecoder: age-out + attention per layer, eager and
    graph-captured, as one fused call per layer or as age-out + attention.
    cap=128 with a 126-token middle runs into the capacity: later steps attend
    the unchanged tiers and drop the new token.  L=1 chains each step's call
    directly after the same layer's previous call while the middle grows from
    126 across the 128-token unit boundary.  The stored tiers (codes,
    scales, ring) must match the oracle bit for bit."""
    from fade_b200.decoder import TieredDecoder

    dt = "bf16"
    B, Hq, Hkv, D = 2, 8, 2, 128
    dec = TieredDecoder(L, B, Hq, Hkv, D, dtype=torch.bfloat16, n_sink=4, recent_window=64, mid_capacity=cap,
                        fused=fused)
    cap_r = -(-cap // 128) * 128
    ks_np, vs_np = [], []
    for l in range(L):
        k = seeded_outliers((B, Hkv, S, D), 100 + l, dt)
        v = seeded_outliers((B, Hkv, S, D), 200 + l, dt)
        dec.load_prompt(l, np_to_dt_tensor(k, dt), np_to_dt_tensor(v, dt))
        ks_np.append(k)
        vs_np.append(v)
    rng = np.random.default_rng(4)
    state = []
    for l in range(L):
        k, v = ks_np[l], vs_np[l]
        kp, ks = oq.quant_k_int4(k[:, :, 4:S - 64], dt)
        vp, vs = oq.quant_v_int4(v[:, :, 4:S - 64], dt)
        state.append({"sink_k": k[:, :, :4], "sink_v": v[:, :, :4], "mid_kq": kp, "mid_ks": ks,
                      "mid_vq": vp, "mid_vs": vs, "ring_k": k[:, :, S - 64:].copy(), "ring_v": v[:, :, S - 64:].copy(),
                      "n": S - 68, "origin": S - 68})
    for step in range(4):
        q = from_bits_dt(rng.standard_normal((L, B, Hq, 1, D)).astype(np.float32), dt)
        kn = from_bits_dt(rng.standard_normal((L, B, Hkv, D)).astype(np.float32), dt)
        vn = from_bits_dt(rng.standard_normal((L, B, Hkv, D)).astype(np.float32), dt)
        if step == 2:
            dec.capture()
        out = t_vals(dec.step(np_to_dt_tensor(q, dt), np_to_dt_tensor(kn, dt), np_to_dt_tensor(vn, dt)))
        for l in range(L):
            s = state[l]
            if s["n"] < cap_r:
                slot = (s["n"] - s["origin"]) % 64
                akp, avp, avs = oq.age_out_int4(s["ring_k"][:, :, slot], s["ring_v"][:, :, slot], s["mid_ks"][:, :, 0],
                                                dt)
                s["mid_kq"] = np.concatenate([s["mid_kq"], akp[:, :, None]], axis=2)
                s["mid_vq"] = np.concatenate([s["mid_vq"], avp[:, :, None]], axis=2)
                s["mid_vs"] = np.concatenate([s["mid_vs"], avs[:, :, None, None]], axis=2)
                s["ring_k"][:, :, slot] = kn[l]
                s["ring_v"][:, :, slot] = vn[l]
                s["n"] += 1
            tiers = {"sink_k": s["sink_k"], "sink_v": s["sink_v"], "int4_kq": s["mid_kq"], "int4_ks": s["mid_ks"],
                     "int4_vq": s["mid_vq"], "int4_vs": s["mid_vs"], "recent_k": s["ring_k"], "recent_v": s["ring_v"]}
            ref = oa.tiered_attention(q[l], tiers, dt)
            assert_attn_close(out[l], ref, dt, TOL[dt])
    assert dec.mid_lengths() == [min(S - 68 + 4, cap_r)] * L
    for l in range(L):
        s, ly = state[l], dec.layers[l]
        n = s["n"]
        np.testing.assert_array_equal(ly.mid_kq[:, :, :n].cpu().numpy(), s["mid_kq"])
        np.testing.assert_array_equal(ly.mid_vq[:, :, :n].cpu().numpy(), s["mid_vq"])
        np.testing.assert_array_equal(t_bits(ly.mid_vs[:, :, :n]), to_bits(s["mid_vs"], dt))
        np.testing.assert_array_equal(t_bits(ly.ring_k), to_bits(s["ring_k"], dt))
        np.testing.assert_array_equal(t_bits(ly.ring_v), to_bits(s["ring_v"], dt))


def test_step_host_graph_matches_device_step(cuda_device):
    """step_host replayed from capture_host (copies overlapping the layers)
    gives the same bits and the same cache state as device-input steps."""
    from fade_b200.decoder import TieredDecoder

    dt = "bf16"
    L, B, Hq, Hkv, D, S = 3, 2, 8, 2, 128, 400
    decs = [TieredDecoder(L, B, Hq, Hkv, D, dtype=torch.bfloat16, n_sink=4, recent_window=64, mid_capacity=512)
            for _ in range(2)]
    for l in range(L):
        k = np_to_dt_tensor(seeded_outliers((B, Hkv, S, D), 300 + l, dt), dt)
        v = np_to_dt_tensor(seeded_outliers((B, Hkv, S, D), 400 + l, dt), dt)
        for d in decs:
            d.load_prompt(l, k, v)
    dev_dec, host_dec = decs
    qh = torch.empty(L, B, Hq, 1, D, dtype=torch.bfloat16).pin_memory()
    kh = torch.empty(L, B, Hkv, D, dtype=torch.bfloat16).pin_memory()
    vh = torch.empty(L, B, Hkv, D, dtype=torch.bfloat16).pin_memory()
    oh = torch.empty(L, B, Hq, 1, D, dtype=torch.bfloat16).pin_memory()
    gen = torch.Generator().manual_seed(7)
    for step in range(4):
        qh.copy_(torch.randn(qh.shape, generator=gen).to(torch.bfloat16))
        kh.copy_(torch.randn(kh.shape, generator=gen).to(torch.bfloat16))
        vh.copy_(torch.randn(vh.shape, generator=gen).to(torch.bfloat16))
        if step == 1:
            dev_dec.capture()
            host_dec.capture_host(qh, kh, vh, oh)
        ref = dev_dec.step(qh.to(cuda_device), kh.to(cuda_device), vh.to(cuda_device)).clone()
        host_dec.step_host(qh, kh, vh, oh)
        torch.cuda.synchronize()
        assert torch.equal(oh, ref.cpu()), step
    assert host_dec.mid_lengths() == dev_dec.mid_lengths() == [S - 68 + 4] * L


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("Sq,Sk", [(1, 301), (5, 301), (7, 1000)])
def test_fused_int4_sdpa_dropin(cuda_device, causal, Sq, Sk):
    """fused_int4_sdpa (fade/kernels/fused_int4_attn.py:277-342): S_q >= 1,
    GQA, fp16, with the reference kernel's causal mask (query m attends keys
    0..m) against the oracle's dequant + SDPA with that mask."""
    from fade_b200.attention import fused_int4_sdpa

    dt = "f16"
    B, Hq, Hkv, D = 2, 8, 2, 128
    k = seeded_outliers((B, Hkv, Sk, D), 71, dt)
    v = seeded_outliers((B, Hkv, Sk, D), 72, dt)
    kp, ks = oq.quant_k_int4(k, dt)
    vp, vs = oq.quant_v_int4(v, dt)
    q = from_bits_dt(np.random.default_rng(73).standard_normal((B, Hq, Sq, D)).astype(np.float32), dt)
    out = t_vals(fused_int4_sdpa(np_to_dt_tensor(q, dt), torch.from_numpy(kp).cuda(), np_to_dt_tensor(ks, dt),
                                 torch.from_numpy(vp).cuda(), np_to_dt_tensor(vs, dt), is_causal=causal))
    kd, vd = oq.dequant_int4(kp, ks, dt), oq.dequant_int4(vp, vs, dt)
    # The middle tier rounds P to fp16 for the PV product; with a handful of
    # keys (the first causal rows) single weights dominate and that rounding
    # reaches 2 output ulps.  The reference's Triton kernel feeds P to tl.dot
    # in fp32, i.e. TF32 on the tensor cores: the same precision class.
    for m in range(Sq):
        n = min(m + 1, Sk) if causal else Sk
        ref = oa.sdpa(q[:, :, m:m + 1], kd[:, :, :n], vd[:, :, :n])
        assert_attn_close(out[:, :, m:m + 1], ref, dt, TOL[dt], ulps=2 if n <= 16 else 1)


def test_paged_int4_middle(cuda_device):
    """A paged middle (128-token pages scattered over a shared pool, a block
    table per (b, h), ragged lengths) gives the oracle's attention, and the
    same result as the contiguous layout of the same tokens."""
    from fade_b200.attention import FPTier, Int4Tier, tiered_decode_attention

    dt = "bf16"
    B, Hq, Hkv, D, cap = 3, 8, 2, 128, 1024
    lens = np.array([1000, 130, 640], dtype=np.int32)
    x = seeded_outliers((B, Hkv, cap, D), 81, dt)
    v = seeded_outliers((B, Hkv, cap, D), 82, dt)
    kp = np.zeros((B, Hkv, cap, D // 2), np.uint8)
    vp = np.zeros_like(kp)
    ks = np.zeros((B, Hkv, 1, D), np.float32)
    vs = np.zeros((B, Hkv, cap, 1), np.float32)
    for b in range(B):
        n = lens[b]
        kp[b:b + 1, :, :n], ks[b:b + 1] = oq.quant_k_int4(x[b:b + 1, :, :n], dt)
        vp[b:b + 1, :, :n], vs[b:b + 1, :, :n] = oq.quant_v_int4(v[b:b + 1, :, :n], dt)
    ppr = cap // 128
    rng = np.random.default_rng(5)
    n_pages = B * Hkv * ppr + 3
    perm = rng.permutation(n_pages)[:B * Hkv * ppr].astype(np.int32)     # scattered, some pool pages unused
    table = perm.reshape(B * Hkv, ppr)
    pool_k = np.zeros((n_pages * 128, D // 2), np.uint8)
    pool_v = np.zeros_like(pool_k)
    pool_s = np.full((n_pages * 128, 1), 0.0, np.float32)
    for z in range(B * Hkv):
        b, h = divmod(z, Hkv)
        for pg in range(ppr):
            r = table[z, pg] * 128
            pool_k[r:r + 128] = kp[b, h, pg * 128:(pg + 1) * 128]
            pool_v[r:r + 128] = vp[b, h, pg * 128:(pg + 1) * 128]
            pool_s[r:r + 128] = vs[b, h, pg * 128:(pg + 1) * 128]
    q = from_bits_dt(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    sink = seeded_outliers((B, Hkv, 4, D), 83, dt)
    qt = np_to_dt_tensor(q, dt)
    lens_t = torch.from_numpy(lens).cuda()
    fp = FPTier(np_to_dt_tensor(sink, dt), np_to_dt_tensor(sink, dt))
    paged = Int4Tier(torch.from_numpy(pool_k).cuda(), np_to_dt_tensor(ks, dt), torch.from_numpy(pool_v).cuda(),
                     np_to_dt_tensor(pool_s, dt), lens=lens_t, max_len=cap,
                     page_table=torch.from_numpy(table).cuda())
    dense = Int4Tier(torch.from_numpy(kp).cuda(), np_to_dt_tensor(ks, dt), torch.from_numpy(vp).cuda(),
                     np_to_dt_tensor(vs, dt), lens=lens_t, max_len=cap)
    units = np.repeat(-(-lens // 128), Hkv)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(units)]).astype(np.int32)).cuda()
    out_p = t_vals(tiered_decode_attention(qt, [fp, paged], cu_units=cu))
    out_d = t_vals(tiered_decode_attention(qt, [fp, dense], cu_units=cu))
    np.testing.assert_array_equal(out_p, out_d)      # same tokens, same order of work
    for b in range(B):
        n = lens[b]
        t = {"sink_k": sink[b:b + 1], "sink_v": sink[b:b + 1], "int4_kq": kp[b:b + 1, :, :n],
             "int4_ks": ks[b:b + 1], "int4_vq": vp[b:b + 1, :, :n], "int4_vs": vs[b:b + 1, :, :n]}
        assert_attn_close(out_p[b:b + 1], oa.tiered_attention(q[b:b + 1], t, dt), dt, TOL[dt])
