"""Generate the golden fixtures in tests/golden/ by running the REFERENCE.

Usage (needs the reference checkout; it is not present on the GPU box, which
only reads the committed .npz files):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/fade-reference

Every fixture stores raw storage bits (uint16 for fp16/bf16) so comparisons
are bit-exact.  Inputs are seeded synthetic tensors with the shapes and value
distributions of the benchmark configs (N(0,1) with per-head outlier
channels scaled x8, keys RoPE'd at their positions).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(OUT))
from inputs import CFG3, CFG4, cfg3_inputs, cfg4_inputs, checksum, outlier_tensor  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float32:
        return t.contiguous().numpy().view(np.uint32).copy()
    return t.contiguous().numpy().copy()


def rope_schemes(ref: str) -> None:
    """cos/sin tables of every RoPE scheme family (fade/rope.py)."""
    sys.path.insert(0, ref)
    from fade import rope as R

    schemes = {
        "vanilla": R.Vanilla(theta=5e5, head_dim=128),
        "linear": R.LinearScaled(theta=1e4, head_dim=64, factor=4.0),
        "llama3": R.Llama3(theta=5e5, head_dim=128, factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                           original_max_position_embeddings=8192),
        "ntk": R.NtkAware(theta=1e4, head_dim=64, factor=2.0),
        "yarn": R.Yarn(theta=1e6, head_dim=128, factor=4.0, original_max_position_embeddings=32768),
        "proportional": R.Proportional(theta=1e4, head_dim=64, partial_rotary_factor=0.5),
        "mrope": R.MRope(theta=1e6, head_dim=128, partial_rotary_factor=1.0, mrope_section=[16, 24, 24]),
        "norope": R.NoRope(theta=1e4, head_dim=64),
    }
    pos = torch.tensor([0, 1, 2, 3, 17, 255, 4095, 8191, 32767, 100000])
    out = {"positions": pos.numpy()}
    for name, sc in schemes.items():
        for dn, dt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
            c, s_ = sc.compute_cos_sin(pos, torch.device("cpu"), model_dtype=dt)
            out[f"{name}_{dn}_cos"] = c[0, 0].numpy()
            out[f"{name}_{dn}_sin"] = s_[0, 0].numpy()
    np.savez_compressed(OUT / "rope_schemes.npz", **out)


def cache_perseq(ref: str) -> None:
    """Per-sequence tier assignment (fade/cache.py:1059-1230): two rows with
    different evictions, then the stored FP16 / INT4 tiers and positions."""
    sys.path.insert(0, ref)
    from fade.cache import TIER_EVICT, TIER_FP16, TIER_INT4, TieredKVCache
    from fade.rope import Vanilla

    gen = torch.Generator().manual_seed(5)
    B, H, D, S = 2, 2, 64, 160
    dt = torch.float16
    scheme = Vanilla(theta=1e4, head_dim=D)
    c, s_ = scheme.compute_cos_sin(torch.arange(S), torch.device("cpu"), model_dtype=dt)
    k = TieredKVCache._apply_rope(outlier_tensor((B, H, S, D), gen).to(dt), c, s_)
    v = outlier_tensor((B, H, S, D), gen).to(dt)
    cache = TieredKVCache(n_sink=4, recent_window=16, int4_budget=80, dtype=dt, head_dim=D, rope_scheme=scheme)
    cache.update(k, v, 0)
    t = torch.full((B, S), TIER_INT4, dtype=torch.long)
    t[:, :4] = TIER_FP16
    t[:, S - 16:] = TIER_FP16
    t[0, 10:40] = TIER_EVICT          # row 0 loses 30 tokens
    t[1, 50:60] = TIER_EVICT          # row 1 loses 10
    cache.apply_tier_assignment_per_sequence(0, t)
    st = cache._layers[0]
    out = {"k": bits(k), "v": bits(v), "tiers": t.numpy(),
           "fp16_k": bits(st.fp16_k), "fp16_v": bits(st.fp16_v), "fp16_pos": st.fp16_pos.numpy(),
           "int4_kq": st.int4_kq.numpy(), "int4_ks": bits(st.int4_ks), "int4_vq": st.int4_vq.numpy(),
           "int4_vs": bits(st.int4_vs), "int4_pos": st.int4_pos.numpy(),
           "next_position": np.int64(st.next_position), "sink_count": np.int64(st.sink_count)}
    np.savez_compressed(OUT / "cache_perseq.npz", **out)


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    import torch.nn.functional as F
    from fade.cache import TieredKVCache
    from fade.policy import _assign_one_layer
    from fade.quant import quant_k_int2, quant_k_int4, quant_v_int2, quant_v_int4
    from fade.rope import Vanilla
    from fade.rotated_quant import (_random_orthogonal, rotated_dequant_k, rotated_dequant_v,
                                    rotated_quant_k, rotated_quant_v)
    from fade.backends import RotatedINT4Backend

    dts = {"f16": torch.float16, "bf16": torch.bfloat16}

    # ------------------------------------------------------------------ quant
    g = torch.Generator().manual_seed(1234)
    q = {}
    for name, dt in dts.items():
        x = outlier_tensor((2, 3, 37, 64), g).to(dt)
        x[0, 0, :, 5] = 0          # an all-zero channel (K scale 0 in fp16)
        x[0, 1, 7, :] = 0          # an all-zero token (V scale 0 in fp16)
        x[1, 0, :, 9] *= 1e-6      # tiny channel (subnormal range in fp16)
        x[1, 2, 3, :] *= 1e-6      # tiny token
        x[1, 1, :, 11] *= 300.0    # large channel
        kp, ks = quant_k_int4(x)
        vp, vs = quant_v_int4(x)
        q[f"{name}_x"] = bits(x)
        q[f"{name}_k_packed"] = kp.numpy()
        q[f"{name}_k_scale"] = bits(ks)
        q[f"{name}_v_packed"] = vp.numpy()
        q[f"{name}_v_scale"] = bits(vs)
        x2 = outlier_tensor((2, 2, 128, 64), g).to(dt)
        x2[0, 1, :32, 3] = 0
        q[f"{name}_x2"] = bits(x2)
        for G in (32, 64):
            kq, kss = quant_k_int2(x2, group_size=G)
            vq, vss = quant_v_int2(x2, group_size=G)
            q[f"{name}_k2_g{G}_codes"] = kq.numpy()
            q[f"{name}_k2_g{G}_scale"] = bits(kss)
            q[f"{name}_v2_g{G}_codes"] = vq.numpy()
            q[f"{name}_v2_g{G}_scale"] = bits(vss)
    np.savez_compressed(OUT / "quant.npz", **q)

    # --------------------------------------------------------------- rotated
    r = {}
    for D in (64, 128):
        R = _random_orthogonal(D, 42)
        r[f"R{D}"] = R.numpy()
        for name, dt in dts.items():
            x = outlier_tensor((1, 2, 40, D), g).to(dt)
            r[f"{name}_D{D}_x"] = bits(x)
            for b in (2, 4):
                kp, ks = rotated_quant_k(x, R, bits=b)
                vp, vs = rotated_quant_v(x, R, bits=b)
                r[f"{name}_D{D}_b{b}_k_packed"] = kp.numpy()
                r[f"{name}_D{D}_b{b}_k_scale"] = bits(ks)
                r[f"{name}_D{D}_b{b}_v_packed"] = vp.numpy()
                r[f"{name}_D{D}_b{b}_v_scale"] = bits(vs)
                r[f"{name}_D{D}_b{b}_k_deq"] = bits(rotated_dequant_k(kp, ks, R, bits=b, dtype=dt))
                r[f"{name}_D{D}_b{b}_v_deq"] = bits(rotated_dequant_v(vp, vs, R, bits=b, dtype=dt))
    np.savez_compressed(OUT / "rotated.npz", **r)

    # ------------------------------------------------------------------ rope
    ro = {}
    for name, dt in dts.items():
        S, D = 48, 64
        scheme = Vanilla(theta=1e6, head_dim=D)
        pos = torch.arange(S)
        keep = torch.tensor([0, 1, 2, 3, 7, 8, 15, 20, 21, 30, 40, 44, 45, 46, 47])
        new_pos = torch.arange(keep.numel())
        c_old, s_old = scheme.compute_cos_sin(pos, torch.device("cpu"), model_dtype=dt)
        c_new, s_new = scheme.compute_cos_sin(new_pos, torch.device("cpu"), model_dtype=dt)
        k_pre = torch.randn(1, 2, S, D, generator=g).to(dt)
        k = TieredKVCache._apply_rope(k_pre, c_old, s_old)
        k_un = TieredKVCache._inverse_rope(k, c_old, s_old)
        out = TieredKVCache._apply_rope(k_un.index_select(-2, keep).contiguous(), c_new, s_new)
        ro[f"{name}_k"] = bits(k)
        ro[f"{name}_keep"] = keep.numpy()
        ro[f"{name}_cos_old"] = c_old[0, 0].numpy()
        ro[f"{name}_sin_old"] = s_old[0, 0].numpy()
        ro[f"{name}_cos_new"] = c_new[0, 0].numpy()
        ro[f"{name}_sin_new"] = s_new[0, 0].numpy()
        ro[f"{name}_out"] = bits(out)
    np.savez_compressed(OUT / "rope.npz", **ro)

    # ------------------------------------------- decode: config 1 (Qwen-0.5B)
    gen = torch.Generator().manual_seed(1)
    B, Hq, Hkv, D, S = 1, 14, 2, 64, 2048
    dt = torch.float16
    scheme = Vanilla(theta=1e6, head_dim=D)
    k_pre = outlier_tensor((B, Hkv, S, D), gen)
    v = outlier_tensor((B, Hkv, S, D), gen).to(dt)
    c, s = scheme.compute_cos_sin(torch.arange(S), torch.device("cpu"), model_dtype=dt)
    k = TieredKVCache._apply_rope(k_pre.to(dt), c, s)
    qv = torch.randn(B, Hq, 1, D, generator=gen).to(dt)
    cache = TieredKVCache(n_sink=4, recent_window=64, int4_budget=None, dtype=dt, rope_theta=1e6, head_dim=D)
    cache.update(k, v, 0)
    tiers = _assign_one_layer(S, torch.arange(S, dtype=torch.float32), 4, 64, None, 0)
    cache.apply_tier_assignment(0, tiers)
    st = cache._layers[0]
    K, V = cache._materialize(0)
    out = F.scaled_dot_product_attention(qv, K, V, enable_gqa=True)
    out32 = F.scaled_dot_product_attention(qv.float(), K.float(), V.float(), enable_gqa=True)
    d1 = {
        "q": bits(qv), "k_roped": bits(k), "v": bits(v),
        "sink_k": bits(st.sink_k), "sink_v": bits(st.sink_v),
        "recent_k": bits(st.fp16_k), "recent_v": bits(st.fp16_v),
        "int4_kq": st.int4_kq.numpy(), "int4_ks": bits(st.int4_ks),
        "int4_vq": st.int4_vq.numpy(), "int4_vs": bits(st.int4_vs),
        "out_ref": bits(out), "out_ref32": bits(out32),
    }
    np.savez_compressed(OUT / "decode_cfg1.npz", **d1)

    # ------------------- decode: config 3 shape, small (K INT4, V INT2, evict)
    gen = torch.Generator().manual_seed(3)
    B, Hq, Hkv, D, S = 2, 8, 2, 128, 512
    dt = torch.float16
    scheme = Vanilla(theta=1e6, head_dim=D)
    k_pre = outlier_tensor((B, Hkv, S, D), gen)
    v = outlier_tensor((B, Hkv, S, D), gen).to(dt)
    c, s = scheme.compute_cos_sin(torch.arange(S), torch.device("cpu"), model_dtype=dt)
    k = TieredKVCache._apply_rope(k_pre.to(dt), c, s)
    qv = torch.randn(B, Hq, 1, D, generator=gen).to(dt)
    cache = TieredKVCache(n_sink=4, recent_window=64, int4_budget=100, dtype=dt, rope_theta=1e6,
                          head_dim=D, middle_v_bits=2, rope_scheme=scheme)
    cache.update(k, v, 0)
    torch.manual_seed(3)
    scores = torch.distributions.Dirichlet(torch.full((S,), 0.1)).sample((Hkv,)).sum(0)
    tiers = _assign_one_layer(S, scores, 4, 64, 100, 0)
    cache.apply_tier_assignment(0, tiers)
    st = cache._layers[0]
    K, V = cache._materialize(0)
    out = F.scaled_dot_product_attention(qv, K, V, enable_gqa=True)
    out32 = F.scaled_dot_product_attention(qv.float(), K.float(), V.float(), enable_gqa=True)
    d3 = {
        "q": bits(qv), "k_roped": bits(k), "v": bits(v), "tiers": tiers.numpy(),
        "sink_k": bits(st.sink_k), "sink_v": bits(st.sink_v),
        "recent_k": bits(st.fp16_k), "recent_v": bits(st.fp16_v),
        "int4_kq": st.int4_kq.numpy(), "int4_ks": bits(st.int4_ks),
        "int4_vq2": st.int4_vq.numpy(), "int4_vs2": bits(st.int4_vs),
        "n_mid": np.int64(st.int4_pos.shape[0]), "next_position": np.int64(st.next_position),
        "out_ref": bits(out), "out_ref32": bits(out32),
    }
    np.savez_compressed(OUT / "decode_cfg3_small.npz", **d3)

    # --------------------- decode: rotated 2-bit backend (config 4 shape), bf16
    gen = torch.Generator().manual_seed(4)
    B, Hq, Hkv, D, S = 1, 7, 1, 128, 300
    dt = torch.bfloat16
    k = outlier_tensor((B, Hkv, S, D), gen).to(dt)
    v = outlier_tensor((B, Hkv, S, D), gen).to(dt)
    qv = torch.randn(B, Hq, 1, D, generator=gen).to(dt)
    backend = RotatedINT4Backend(head_dim=D, bits=2, seed=42)
    cache = TieredKVCache(n_sink=4, recent_window=64, int4_budget=None, dtype=dt, head_dim=D,
                          quant_backend=backend)
    cache.update(k, v, 0)
    tiers = _assign_one_layer(S, torch.arange(S, dtype=torch.float32), 4, 64, None, 0)
    cache.apply_tier_assignment(0, tiers)
    st = cache._layers[0]
    K, V = cache._materialize(0)
    out = F.scaled_dot_product_attention(qv, K, V, enable_gqa=True)
    out32 = F.scaled_dot_product_attention(qv.float(), K.float(), V.float(), enable_gqa=True)
    d4 = {
        "q": bits(qv), "k": bits(k), "v": bits(v), "R": _random_orthogonal(D, 42).numpy(),
        "sink_k": bits(st.sink_k), "sink_v": bits(st.sink_v),
        "recent_k": bits(st.fp16_k), "recent_v": bits(st.fp16_v),
        "rot_kq": st.backend_k["packed"].numpy(), "rot_ks": bits(st.backend_k["scale"]),
        "rot_vq": st.backend_v["packed"].numpy(), "rot_vs": bits(st.backend_v["scale"]),
        "out_ref": bits(out), "out_ref32": bits(out32),
    }
    np.savez_compressed(OUT / "decode_rot_small.npz", **d4)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


def decode_cfg3_g32(ref: str) -> None:
    """Config 3 at the benchmark configuration's settings (batch sliced to 1): H2O survivors of a
    4096-token prompt (_assign_one_layer, budget 400) through the reference's
    evicting apply_tier_assignment (un-RoPE / re-RoPE), K INT4, V grouped INT2
    with group 32 (quant_v_int2(pad_to_group(v, 32), 32)), then the reference's
    dequant + SDPA over sink | middle | recent."""
    sys.path.insert(0, ref)
    import torch.nn.functional as F
    from fade.cache import TIER_FP16, TIER_INT4, TieredKVCache
    from fade.policy import _assign_one_layer
    from fade.quant import dequant_int4, dequant_v_int2, pad_to_group, quant_v_int2
    from fade.rope import Vanilla

    c = CFG3
    dt = torch.float16
    scheme = Vanilla(theta=c["theta"], head_dim=c["D"])
    k, v, q, scores = cfg3_inputs(lambda pos: scheme.compute_cos_sin(pos, torch.device("cpu"), model_dtype=dt))
    cache = TieredKVCache(n_sink=c["n_sink"], recent_window=c["recent"], int4_budget=c["budget"], dtype=dt,
                          rope_theta=c["theta"], head_dim=c["D"], rope_scheme=scheme)
    cache.update(k, v, 0)
    tiers = _assign_one_layer(c["S"], scores, c["n_sink"], c["recent"], c["budget"], 0)
    cache.apply_tier_assignment(0, tiers)
    st = cache._layers[0]
    keep = tiers != 3
    kept = tiers[keep]
    v_mid = v[:, :, keep.nonzero().squeeze(-1)][:, :, (kept == TIER_INT4).nonzero().squeeze(-1)]
    n_mid = v_mid.shape[2]
    vq, vs = quant_v_int2(pad_to_group(v_mid, c["group"])[0], group_size=c["group"])
    k_mid = dequant_int4(st.int4_kq, st.int4_ks, dtype=dt)
    v_deq = dequant_v_int2(vq, vs, group_size=c["group"], dtype=dt)[:, :, :n_mid]
    K = torch.cat([st.sink_k, k_mid, st.fp16_k], dim=2)
    V = torch.cat([st.sink_v, v_deq, st.fp16_v], dim=2)
    out32 = F.scaled_dot_product_attention(q.float(), K.float(), V.float(), enable_gqa=True)
    out = F.scaled_dot_product_attention(q, K, V, enable_gqa=True)
    d = {"k_sum": np.int64(checksum(k)), "v_sum": np.int64(checksum(v)), "q": bits(q), "tiers": tiers.numpy(),
         "sink_k": bits(st.sink_k), "sink_v": bits(st.sink_v), "recent_k": bits(st.fp16_k),
         "recent_v": bits(st.fp16_v), "int4_kq": st.int4_kq.numpy(), "int4_ks": bits(st.int4_ks),
         "v_mid": bits(v_mid), "int2_vq": vq.numpy(), "int2_vs": bits(vs), "n_mid": np.int64(n_mid),
         "out_ref": bits(out), "out_ref32": bits(out32)}
    np.savez_compressed(OUT / "decode_cfg3_g32.npz", **d)


def decode_cfg4_ragged(ref: str) -> None:
    """Config 4 shape: ragged sequences, rotated 2-bit middle.  The reference
    has no batched ragged path, so this is its per-sequence loop: each
    sequence's middle through rotated_quant_k / rotated_quant_v, then
    rotated_dequant + cat(sink, middle, recent) + SDPA."""
    sys.path.insert(0, ref)
    import torch.nn.functional as F
    from fade.rotated_quant import (_random_orthogonal, rotated_dequant_k, rotated_dequant_v,
                                    rotated_quant_k, rotated_quant_v)

    c = CFG4
    R = _random_orthogonal(c["D"], 42)
    lens, seqs, q = cfg4_inputs()
    d = {"lens": np.array(lens, dtype=np.int64), "q": bits(q), "R": R.numpy()}
    ns, nr = c["n_sink"], c["recent"]
    for i, (k, v) in enumerate(seqs):
        n = k.shape[2]
        kq, ks = rotated_quant_k(k[:, :, ns:n - nr], R, bits=c["bits"])
        vq, vs = rotated_quant_v(v[:, :, ns:n - nr], R, bits=c["bits"])
        kd = rotated_dequant_k(kq, ks, R, bits=c["bits"], dtype=torch.bfloat16)
        vd = rotated_dequant_v(vq, vs, R, bits=c["bits"], dtype=torch.bfloat16)
        K = torch.cat([k[:, :, :ns], kd, k[:, :, n - nr:]], dim=2)
        V = torch.cat([v[:, :, :ns], vd, v[:, :, n - nr:]], dim=2)
        qi = q[i:i + 1]
        d[f"s{i}_k_sum"] = np.int64(checksum(k))
        d[f"s{i}_v_sum"] = np.int64(checksum(v))
        d[f"s{i}_kq"], d[f"s{i}_ks"] = kq.numpy(), bits(ks)
        d[f"s{i}_vq"], d[f"s{i}_vs"] = vq.numpy(), bits(vs)
        d[f"s{i}_out_ref32"] = bits(F.scaled_dot_product_attention(qi.float(), K.float(), V.float(),
                                                                    enable_gqa=True))
        d[f"s{i}_out_ref"] = bits(F.scaled_dot_product_attention(qi, K, V, enable_gqa=True))
    np.savez_compressed(OUT / "decode_cfg4_ragged.npz", **d)


def cache_state(ref: str) -> None:
    """The reference's own checkpoint of a cache (cache_state_dict,
    fade/cache.py:510-559) for the config-1 state: the prompt of
    decode_cfg1.npz through update + apply_tier_assignment, saved with
    torch.save, for loading into fade_b200's TieredKVCache."""
    sys.path.insert(0, ref)
    from fade.cache import TieredKVCache
    from fade.policy import _assign_one_layer

    g = np.load(OUT / "decode_cfg1.npz")
    k = torch.from_numpy(g["k_roped"].view(np.int16)).view(torch.float16)
    v = torch.from_numpy(g["v"].view(np.int16)).view(torch.float16)
    S = k.shape[2]
    cache = TieredKVCache(n_sink=4, recent_window=64, int4_budget=None, dtype=torch.float16, rope_theta=1e6,
                          head_dim=64)
    cache.update(k, v, 0)
    cache.apply_tier_assignment(0, _assign_one_layer(S, torch.arange(S, dtype=torch.float32), 4, 64, None, 0))
    torch.save(cache.cache_state_dict(), OUT / "cache_state_cfg1.pt")


if __name__ == "__main__":
    import os

    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref_path = args[0] if args else os.environ.get("FADE_REFERENCE_PATH")
    if not ref_path:
        raise SystemExit("usage: make_golden.py <path to the reference checkout> [--only-rope-schemes|--only-cache-perseq|--only-cfg3-cfg4|--only-cache-state]")
    if "--only-rope-schemes" in sys.argv:
        rope_schemes(ref_path)
    elif "--only-cache-state" in sys.argv:
        cache_state(ref_path)
    elif "--only-cfg3-cfg4" in sys.argv:
        decode_cfg3_g32(ref_path)
        decode_cfg4_ragged(ref_path)
        cache_state(ref_path)
    elif "--only-cache-perseq" in sys.argv:
        cache_perseq(ref_path)
    else:
        main(ref_path)
        rope_schemes(ref_path)
        cache_perseq(ref_path)
        decode_cfg3_g32(ref_path)
        decode_cfg4_ragged(ref_path)
        cache_state(ref_path)
