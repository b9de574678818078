"""TieredKVCache / create_tiered_cache on the GPU against the reference's own
cache states (fixtures made by running the reference: tests/golden/) and
against transformers' SDPA path on the same model."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import assert_attn_close, t_bits, t_from_bits, t_vals
from oracle import quant as oq
from oracle.numerics import to_bits

pytestmark = pytest.mark.gpu
TOL = {"f16": 2e-3, "bf16": 1e-2}


def _tiers(S, n_sink=4, recent=64):
    from fade_b200.cache import TIER_FP16, TIER_INT4

    t = torch.full((S,), TIER_INT4, dtype=torch.long)
    t[:n_sink] = TIER_FP16
    t[S - recent:] = TIER_FP16
    return t


def _eq(t, ref_bits, what):
    np.testing.assert_array_equal(t_bits(t), ref_bits, err_msg=what)


def _device_tables(cache, S, n_kept, D, device):
    """cos/sin exactly as the cache (and the reference's RopeScheme.compute_cos_sin,
    fade/rope.py:72-93) builds them: torch ops on the cache's device."""
    pos = torch.arange(S, device=device)
    c, s = cache._compute_cos_sin(torch.cat([pos, torch.arange(n_kept, device=device)]), device)
    c, s = c.reshape(-1, D).float().cpu().numpy(), s.reshape(-1, D).float().cpu().numpy()
    return c[:S], s[:S], c[S:], s[S:]


def _oracle_survivors(cache, k_bits, tiers_row, dt, device):
    """The reference's evicting branch (fade/cache.py:914-935) restated by the
    oracle with the cache's device tables: re-RoPE'd K of the survivors
    [B,H,n_kept,D] and their tiers."""
    from oracle import rope as orope
    from oracle.numerics import from_bits

    k = from_bits(k_bits, dt)
    D, S = k.shape[-1], k.shape[2]
    keep = np.nonzero(tiers_row != 3)[0]
    co, so, cn, sn = _device_tables(cache, S, len(keep), D, device)
    return orope.rerope_gather(k, keep, co, so, cn, sn, dt), tiers_row[keep]


def test_cache_cfg1_tiers_and_decode(cuda_device):
    """Config-1 shape, no eviction: tiers bit-exact, fused decode vs the reference's SDPA."""
    from fade_b200.cache import TieredKVCache

    g = golden("decode_cfg1")
    k, v, q = t_from_bits(g["k_roped"], "f16"), t_from_bits(g["v"], "f16"), t_from_bits(g["q"], "f16")
    S = k.shape[2]
    cache = TieredKVCache(n_sink=4, recent_window=64, dtype=torch.float16, rope_theta=1e6, head_dim=64)
    K0, V0 = cache.update(k, v, 0)
    assert torch.equal(K0, k) and torch.equal(V0, v) and cache.get_seq_length(0) == S
    cache.apply_tier_assignment(0, _tiers(S))
    st = cache._layers[0]
    _eq(st.sink_k, g["sink_k"], "sink_k")
    _eq(st.sink_v, g["sink_v"], "sink_v")
    _eq(st.fp16_k, g["recent_k"], "recent_k")
    _eq(st.fp16_v, g["recent_v"], "recent_v")
    np.testing.assert_array_equal(st.int4_kq.cpu().numpy(), g["int4_kq"])
    np.testing.assert_array_equal(st.int4_vq.cpu().numpy(), g["int4_vq"])
    _eq(st.int4_ks, g["int4_ks"], "int4_ks")
    _eq(st.int4_vs, g["int4_vs"], "int4_vs")
    assert cache.get_seq_length(0) == S
    out = cache.decode_attention(0, q)
    assert_attn_close(t_vals(out), t_vals(t_from_bits(g["out_ref32"], "f32")), "f16", TOL["f16"])
    # the materialised path (update with a new token) keeps working after reassignment
    K, V = cache._materialize(0)
    assert K.shape[2] == S


def test_cache_cfg3_eviction_k4v2(cuda_device):
    """Config-3 shape: H2O tiers with eviction (re-RoPE), K INT4 + V grouped INT2."""
    from fade_b200.cache import TieredKVCache
    from fade_b200.rope import Vanilla

    g = golden("decode_cfg3_small")
    k, v, q = t_from_bits(g["k_roped"], "f16"), t_from_bits(g["v"], "f16"), t_from_bits(g["q"], "f16")
    D = k.shape[-1]
    cache = TieredKVCache(n_sink=4, recent_window=64, int4_budget=100, dtype=torch.float16, rope_theta=1e6,
                          head_dim=D, middle_v_bits=2, rope_scheme=Vanilla(theta=1e6, head_dim=D))
    cache.update(k, v, 0)
    cache.apply_tier_assignment(0, torch.from_numpy(g["tiers"]))
    st = cache._layers[0]
    assert st.next_position == int(g["next_position"]) and st.int4_pos.shape[0] == int(g["n_mid"])
    # Values and V codes are not re-RoPE'd: bit-exact with the reference run.
    _eq(st.sink_v, g["sink_v"], "sink_v")
    _eq(st.fp16_v, g["recent_v"], "recent_v")
    np.testing.assert_array_equal(st.int4_vq.cpu().numpy(), g["int4_vq2"])
    _eq(st.int4_vs, g["int4_vs2"], "int4_vs (grouped INT2)")
    # Re-RoPE'd K: the reference builds its cos/sin tables on the cache's
    # device.  The fixture ran on the CPU, whose torch cos/sin can differ from
    # the CUDA ones by an ulp, so against the fixture K is exact or one ulp off.
    # Against the reference's arithmetic on the tables of THIS cache's device
    # (oracle re-RoPE + oracle quantiser) every stored K bit and code is exact.
    kk, kt = _oracle_survivors(cache, g["k_roped"], g["tiers"], "f16", k.device)
    fp = kk[:, :, kt == 0]
    _eq(st.sink_k, to_bits(fp[:, :, :4], "f16"), "sink_k vs oracle")
    _eq(st.fp16_k, to_bits(fp[:, :, 4:], "f16"), "recent_k vs oracle")
    kq, ks = oq.quant_k_int4(kk[:, :, kt == 1], "f16")
    np.testing.assert_array_equal(st.int4_kq.cpu().numpy(), kq)
    _eq(st.int4_ks, to_bits(ks, "f16"), "int4_ks vs oracle")
    for name, ref in (("sink_k", "sink_k"), ("fp16_k", "recent_k")):
        assert np.abs(t_bits(getattr(st, name)).astype(np.int32) - g[ref].astype(np.int32)).max() <= 1, name
    out = cache.decode_attention(0, q)
    assert_attn_close(t_vals(out), t_vals(t_from_bits(g["out_ref32"], "f32")), "f16", TOL["f16"])


def test_cache_rotated_backend(cuda_device):
    """Config-4 shape: rotated 2-bit backend; the fused kernel reads its codes directly."""
    from fade_b200.backends import RotatedINT4Backend
    from fade_b200.cache import TieredKVCache

    g = golden("decode_rot_small")
    k, v, q = t_from_bits(g["k"], "bf16"), t_from_bits(g["v"], "bf16"), t_from_bits(g["q"], "bf16")
    D, S = k.shape[-1], k.shape[2]
    cache = TieredKVCache(n_sink=4, recent_window=64, dtype=torch.bfloat16, head_dim=D,
                          quant_backend=RotatedINT4Backend(head_dim=D, bits=2, seed=42))
    cache.update(k, v, 0)
    cache.apply_tier_assignment(0, _tiers(S))
    st = cache._layers[0]
    _eq(st.sink_k, g["sink_k"], "sink_k")
    _eq(st.fp16_v, g["recent_v"], "recent_v")
    for ours, ref in ((st.backend_k["packed"], "rot_kq"), (st.backend_v["packed"], "rot_vq")):
        assert (ours.cpu().numpy() != g[ref]).mean() < 0.004, ref
    out = cache.decode_attention(0, q)
    assert_attn_close(t_vals(out), t_vals(t_from_bits(g["out_ref32"], "f32")), "bf16", TOL["bf16"], ulps=2,
                      additive=True)


def test_cache_per_sequence_assignment(cuda_device):
    """Per-row tiers with different evictions: stored tiers as the reference's."""
    from fade_b200.cache import TieredKVCache
    from fade_b200.rope import Vanilla

    g = golden("cache_perseq")
    k, v = t_from_bits(g["k"], "f16"), t_from_bits(g["v"], "f16")
    D = k.shape[-1]
    cache = TieredKVCache(n_sink=4, recent_window=16, int4_budget=80, dtype=torch.float16, head_dim=D,
                          rope_scheme=Vanilla(theta=1e4, head_dim=D))
    cache.update(k, v, 0)
    cache.apply_tier_assignment_per_sequence(0, torch.from_numpy(g["tiers"]))
    st = cache._layers[0]
    assert st.next_position == int(g["next_position"]) and st.sink_count == int(g["sink_count"])
    np.testing.assert_array_equal(st.fp16_pos.cpu().numpy(), g["fp16_pos"])
    np.testing.assert_array_equal(st.int4_pos.cpu().numpy(), g["int4_pos"])
    _eq(st.fp16_v, g["fp16_v"], "fp16_v")
    np.testing.assert_array_equal(st.int4_vq.cpu().numpy(), g["int4_vq"])
    _eq(st.int4_vs, g["int4_vs"], "int4_vs")
    # Re-RoPE'd K against the reference's arithmetic on this device's tables
    # (see test_cache_cfg3_eviction_k4v2): bit-exact, rows padded with zero
    # tokens to the longest row as the reference does.
    fp_rows, i4_rows = [], []
    for b in range(k.shape[0]):
        kk, kt = _oracle_survivors(cache, g["k"][b:b + 1], g["tiers"][b], "f16", k.device)
        fp_rows.append(kk[:, :, kt == 0])
        i4_rows.append(kk[:, :, kt == 1])

    def pad(rows):
        n = max(r.shape[2] for r in rows)
        return np.concatenate([np.pad(r, ((0, 0), (0, 0), (0, n - r.shape[2]), (0, 0))) for r in rows], axis=0)

    _eq(st.fp16_k, to_bits(pad(fp_rows), "f16"), "fp16_k vs oracle")
    kq, ks = oq.quant_k_int4(pad(i4_rows), "f16")
    np.testing.assert_array_equal(st.int4_kq.cpu().numpy(), kq)
    _eq(st.int4_ks, to_bits(ks, "f16"), "int4_ks vs oracle")
    # against the CPU-run fixture: exact or one ulp (CPU vs CUDA cos/sin)
    assert np.abs(t_bits(st.fp16_k).astype(np.int32) - g["fp16_k"].astype(np.int32)).max() <= 1
    # fused decode over the per-sequence tiers == SDPA over the materialised cache
    q = torch.randn(k.shape[0], 4, 1, D, device=k.device).to(torch.float16)
    out = cache.decode_attention(0, q)
    K, V = cache._materialize(0)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), K.float(), V.float(), enable_gqa=True)
    assert_attn_close(t_vals(out), t_vals(ref), "f16", TOL["f16"])


def test_checkpoint_roundtrip(cuda_device):
    from fade_b200.cache import TieredKVCache

    g = golden("decode_cfg1")
    k, v, q = t_from_bits(g["k_roped"], "f16"), t_from_bits(g["v"], "f16"), t_from_bits(g["q"], "f16")
    a = TieredKVCache(n_sink=4, recent_window=64, dtype=torch.float16, head_dim=64)
    a.update(k, v, 0)
    a.apply_tier_assignment(0, _tiers(k.shape[2]))
    sd = a.cache_state_dict()
    assert sd["layer.0.int4_kq"].device.type == "cpu"
    b = TieredKVCache(n_sink=4, recent_window=64, dtype=torch.float16, head_dim=64)
    b.load_cache_state_dict(sd, device=k.device)
    assert b.get_seq_length(0) == a.get_seq_length(0)
    assert torch.equal(a.decode_attention(0, q), b.decode_attention(0, q))
    st = a._layers[0]
    sinks = st.sink_k.numel() * 2 + st.sink_v.numel() * 2      # storage_bytes() leaves sinks out, as the reference
    assert b.compressed_storage_bytes() == a.compressed_storage_bytes() > 0
    assert a.storage_bytes() == a.compressed_storage_bytes() - sinks


def test_load_reference_checkpoint(cuda_device):
    """A cache_state_dict written by the reference itself (fade/cache.py:
    510-559; tests/golden/cache_state_cfg1.pt) loads into fade_b200's cache:
    the same tiers bit for bit, and the fused decode over them matches the
    reference's SDPA output."""
    from conftest import ROOT
    from fade_b200.cache import TieredKVCache

    sd = torch.load(ROOT / "tests" / "golden" / "cache_state_cfg1.pt", weights_only=True)
    g = golden("decode_cfg1")
    cache = TieredKVCache(n_sink=4, recent_window=64, dtype=torch.float16, rope_theta=1e6, head_dim=64)
    cache.load_cache_state_dict(sd, device=cuda_device)
    st = cache._layers[0]
    _eq(st.sink_k, g["sink_k"], "sink_k")
    _eq(st.fp16_v, g["recent_v"], "recent_v")
    np.testing.assert_array_equal(st.int4_kq.cpu().numpy(), g["int4_kq"])
    np.testing.assert_array_equal(st.int4_vq.cpu().numpy(), g["int4_vq"])
    _eq(st.int4_ks, g["int4_ks"], "int4_ks")
    _eq(st.int4_vs, g["int4_vs"], "int4_vs")
    assert cache.get_seq_length(0) == 2048 and st.next_position == 2048
    out = cache.decode_attention(0, t_from_bits(g["q"], "f16"))
    assert_attn_close(t_vals(out), t_vals(t_from_bits(g["out_ref32"], "f32")), "f16", TOL["f16"])
    # and back: our checkpoint of it carries the reference's keys and values
    sd2 = cache.cache_state_dict()
    for key, val in sd.items():
        if key.startswith("layer.") and isinstance(val, torch.Tensor):
            assert torch.equal(sd2[key].cpu(), val), key


def _tiny_llama(dev):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=256, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, rope_theta=5e5, max_position_embeddings=1024)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(device=dev, dtype=torch.bfloat16).eval()


def test_hf_decode_fused_matches_sdpa(cuda_device):
    """A (random-init) Llama decodes through create_tiered_cache: the fused
    tiered attention gives the logits of transformers' SDPA over the
    materialised cache, before and after an INT4 reassignment."""
    from fade_b200.patch import create_tiered_cache

    dev = torch.device("cuda", 0)
    m_fused, m_ref = _tiny_llama(dev), _tiny_llama(dev)
    m_ref.load_state_dict(m_fused.state_dict())
    c_fused = create_tiered_cache(m_fused, dtype=torch.bfloat16, n_sink=4, recent_window=64)
    c_ref = create_tiered_cache(m_ref, dtype=torch.bfloat16, n_sink=4, recent_window=64, fused_attention=False)
    assert c_fused.fused_decode and not c_ref.fused_decode
    # Every fused attention call is also checked on its own, at the north-star
    # tolerance: against fp32 SDPA over the same cache materialised with the
    # reference's dequantisation (sink | dequant middle | recent).
    checked = []
    fused_call = c_fused.decode_attention

    def checking(layer, query, scaling=None, out=None):
        res = fused_call(layer, query, scaling=scaling, out=out)
        K, V = c_fused._materialize(layer)
        ref = torch.nn.functional.scaled_dot_product_attention(query.float(), K.float(), V.float(),
                                                               scale=scaling, enable_gqa=True)
        checked.append(assert_attn_close(t_vals(res), t_vals(ref), "bf16", TOL["bf16"]))
        return res

    c_fused.decode_attention = checking
    ids = torch.randint(0, 256, (2, 300), generator=torch.Generator().manual_seed(1)).to(dev)
    with torch.no_grad():
        lf = m_fused(input_ids=ids, past_key_values=c_fused, use_cache=True).logits[:, -1]
        lr = m_ref(input_ids=ids, past_key_values=c_ref, use_cache=True).logits[:, -1]
        assert torch.allclose(lf.float(), lr.float(), atol=1e-3)
        nxt = lf.argmax(-1, keepdim=True)
        for step in range(6):
            if step == 2:   # compress the middle of every layer
                for layer in range(2):
                    S = c_fused.get_seq_length(layer)
                    c_fused.apply_tier_assignment(layer, _tiers(S))
                    c_ref.apply_tier_assignment(layer, _tiers(S))
            lf = m_fused(input_ids=nxt, past_key_values=c_fused, use_cache=True).logits[:, -1].float()
            lr = m_ref(input_ids=nxt, past_key_values=c_ref, use_cache=True).logits[:, -1].float()
            err = (lf - lr).abs().max().item()
            assert err < 0.05 * max(1.0, lr.abs().max().item()), (step, err)
            nxt = lr.argmax(-1, keepdim=True)
    assert c_fused.get_seq_length(0) == c_ref.get_seq_length(0) == 306
    assert len(checked) == 2 * 6 and max(checked) <= 1.0
