"""Host-side API (no GPU): FadeConfig, backends, RoPE schemes, create_tiered_cache.

Mirrors the reference's tests of the same surface (tests/test_config.py,
tests/test_backends.py, tests/test_rope.py of fade-kv 1.1.0) and pins the RoPE
tables against fixtures made by running the reference (tests/golden/).
"""

from __future__ import annotations

import types
import warnings

import numpy as np
import pytest
import torch

from conftest import golden


# ------------------------------------------------------------------ config
def test_config_defaults_and_presets():
    from fade_b200.config import FadeConfig

    c = FadeConfig()
    assert (c.phase, c.n_sink, c.recent_window, c.int4_budget, c.int2_budget) == ("1a", 4, 64, None, 0)
    assert (c.eviction_policy, c.reassign_every, c.prefill_track_limit, c.int2_group_size) == ("h2o", 64, 1024, 64)
    assert (c.middle_k_bits, c.middle_v_bits, c.quant_backend) == (4, 4, "int4")
    s, b, a = FadeConfig.safe(), FadeConfig.balanced(), FadeConfig.aggressive()
    assert (s.phase, s.int4_budget) == ("1a", None)
    assert (b.phase, b.int4_budget, b.recent_window) == ("2", 400, 64)
    assert (a.phase, a.int4_budget, a.recent_window) == ("2", 200, 32)
    assert b.to_cache_kwargs() == {"n_sink": 4, "recent_window": 64, "int4_budget": 400, "int2_budget": 0,
                                   "middle_k_bits": 4, "middle_v_bits": 4, "quant_backend": "int4"}
    assert b.with_overrides(int4_budget=10).int4_budget == 10


@pytest.mark.parametrize("kw,msg", [
    (dict(n_sink=-1), "n_sink must be >= 0, got -1"),
    (dict(recent_window=-2), "recent_window must be >= 0, got -2"),
    (dict(phase="2", int4_budget=-1), "int4_budget must be >= 0 or None, got -1"),
    (dict(int2_budget=-1), "int2_budget must be >= 0, got -1"),
    (dict(reassign_every=0), "reassign_every must be >= 1, got 0"),
    (dict(int2_group_size=0), "int2_group_size must be >= 1, got 0"),
    (dict(int4_budget=5), "phase='1a' requires int4_budget=None"),
    (dict(phase="2"), "phase='2' requires at least one of int4_budget / int2_budget > 0"),
    (dict(eviction_policy="lru"), "unknown eviction_policy: 'lru'"),
    (dict(middle_k_bits=3), "middle_k_bits must be 4 or 2, got 3"),
    (dict(middle_v_bits=8), "middle_v_bits must be 4 or 2, got 8"),
])
def test_config_validation(kw, msg):
    from fade_b200.config import FadeConfig

    with pytest.raises(ValueError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        FadeConfig(**kw)


# ---------------------------------------------------------------- backends
def test_get_backend_names_and_errors():
    from fade_b200 import backends as bk

    assert isinstance(bk.get_backend(), bk.SymmetricINT4Backend)
    assert isinstance(bk.get_backend("INT4", head_dim=7), bk.SymmetricINT4Backend)
    r = bk.get_backend("rotated", head_dim=128, bits=2, junk=1)
    assert isinstance(r, bk.RotatedINT4Backend) and (r.head_dim, r.bits, r.seed) == (128, 2, 42)
    assert r.name == "rotated_int2"
    assert isinstance(bk.get_backend("turboquant", head_dim=64), bk.TurboQuantBackend)
    assert isinstance(r, bk.QuantBackend)
    with pytest.raises(ValueError, match="Unknown quant backend 'nope'"):
        bk.get_backend("nope")
    t = bk.get_backend("turbo")
    with pytest.raises(ImportError, match="TurboQuantBackend requires turboquant-kv"):
        t.compress_k(torch.zeros(1, 1, 1, 128))


def test_rotation_matches_reference_seed():
    from fade_b200.backends import RotatedINT4Backend

    R = RotatedINT4Backend(head_dim=128).rotation()
    np.testing.assert_array_equal(R.numpy(), golden("decode_rot_small")["R"])


# -------------------------------------------------------------------- rope
def _schemes():
    from fade_b200 import rope as R

    return {
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


@pytest.mark.parametrize("name", list(_schemes()))
@pytest.mark.parametrize("dn,dt", [("f16", torch.float16), ("bf16", torch.bfloat16)])
def test_rope_tables_match_reference(name, dn, dt):
    g = golden("rope_schemes")
    pos = torch.from_numpy(g["positions"])
    c, s = _schemes()[name].compute_cos_sin(pos, torch.device("cpu"), model_dtype=dt)
    np.testing.assert_array_equal(c[0, 0].numpy(), g[f"{name}_{dn}_cos"])
    np.testing.assert_array_equal(s[0, 0].numpy(), g[f"{name}_{dn}_sin"])


def test_extract_rope_scheme_from_configs():
    from transformers import LlamaConfig

    from fade_b200 import rope as R

    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, rope_theta=5e5,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    sc = R.extract_rope_scheme(cfg)
    assert isinstance(sc, R.Llama3) and sc.factor == 8.0 and sc.head_dim == 128 and sc.theta == 5e5
    plain = types.SimpleNamespace(rope_theta=1e6, hidden_size=64, num_attention_heads=1)
    assert isinstance(R.extract_rope_scheme(plain), R.Vanilla)
    alibi = types.SimpleNamespace(alibi=True, hidden_size=64, num_attention_heads=1)
    assert isinstance(R.extract_rope_scheme(alibi), R.NoRope)
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        odd = types.SimpleNamespace(rope_theta=1e4, rope_scaling={"type": "weird"}, hidden_size=64,
                                    num_attention_heads=1)
        assert isinstance(R.extract_rope_scheme(odd), R.Vanilla)
        assert any("Unknown rope_scaling type" in str(x.message) for x in w)


# ------------------------------------------------------------- the cache
def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, rope_theta=5e5, max_position_embeddings=512)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_create_tiered_cache_binds_model():
    from fade_b200.cache import TieredKVCache
    from fade_b200.config import FadeConfig
    from fade_b200.patch import ATTN_IMPL, create_tiered_cache
    from fade_b200.rope import Vanilla

    model = _tiny_llama()
    cache = create_tiered_cache(model, dtype=torch.bfloat16, config=FadeConfig.balanced(), recent_window=32)
    assert isinstance(cache, TieredKVCache)
    assert (cache.n_sink, cache.recent_window, cache.int4_budget, cache.head_dim) == (4, 32, 400, 32)
    assert isinstance(cache.rope_scheme, Vanilla) and cache.rope_scheme.theta == 5e5
    assert cache.fused_decode and model.config._attn_implementation == ATTN_IMPL
    bound = [m for m in model.modules() if hasattr(m, "_fade_cache")]
    assert len(bound) == 2 and all(m._fade_cache() is cache for m in bound)
    plain = create_tiered_cache(_tiny_llama(), fused_attention=False)
    assert not plain.fused_decode


def test_create_tiered_cache_recurrent_and_mla():
    from transformers.cache_utils import DynamicCache

    from fade_b200.patch import create_tiered_cache

    fake = types.SimpleNamespace(config=types.SimpleNamespace(model_type="mamba"))
    with pytest.warns(RuntimeWarning, match="recurrent architecture"):
        c = create_tiered_cache(fake)
    assert type(c) is DynamicCache
    mla = types.SimpleNamespace(config=types.SimpleNamespace(model_type="deepseek_v3", hidden_size=64,
                                                             num_attention_heads=2, num_hidden_layers=3,
                                                             rope_theta=1e4))
    with pytest.warns(RuntimeWarning, match="Multi-head Latent Attention"):
        c = create_tiered_cache(mla)
    assert not c.is_managed(0) and not c.is_managed(2) and not c.fused_decode


def test_cache_rejects_cpu_tensors_and_bad_shapes():
    from fade_b200.cache import TieredKVCache

    cache = TieredKVCache(dtype=torch.float16)
    with pytest.raises(ValueError, match=r"key_states must be \[B, H, S, D\]"):
        cache.update(torch.zeros(2, 3, 4), torch.zeros(2, 3, 4), 0)
    with pytest.raises(ValueError, match="K/V shape mismatch"):
        cache.update(torch.zeros(1, 2, 3, 8), torch.zeros(1, 2, 4, 8), 0)
    with pytest.raises(RuntimeError, match="There is no CPU path"):
        cache.update(torch.zeros(1, 2, 3, 8), torch.zeros(1, 2, 3, 8), 0)
    assert cache.get_seq_length() == 0 and len(cache) == 0
    assert cache.get_mask_sizes(5) == (5, 0)
    with pytest.raises(NotImplementedError):
        cache.set_codebooks(None)


def test_fade_import_alias():
    """Code importing the reference package by name resolves to fade_b200."""
    import sys

    from fade_b200 import compat

    saved = {k: v for k, v in sys.modules.items() if k == "fade" or k.startswith("fade.")}
    for k in saved:
        del sys.modules[k]
    try:
        compat.install_fade_alias()
        from fade import FadeConfig, TieredKVCache, create_tiered_cache, get_backend  # noqa: F401
        from fade.cache import TIER_INT4
        from fade.kernels.fused_int4_attn import fused_int4_sdpa
        from fade.policy import _assign_one_layer
        from fade.quant import quant_k_int4

        import fade_b200.attention as att
        import fade_b200.cache as cache
        assert TieredKVCache is cache.TieredKVCache and TIER_INT4 == cache.TIER_INT4
        assert fused_int4_sdpa is att.fused_int4_sdpa
        assert FadeConfig.safe().n_sink == 4 and callable(_assign_one_layer) and callable(quant_k_int4)
    finally:
        compat.uninstall_fade_alias()
        sys.modules.update(saved)


def test_assign_counts_match_assign_one_layer():
    """assign_counts gives, from the budgets alone, the FP16 / INT4 / INT2
    counts of _assign_one_layer's tiers (fade/policy.py:232-274)."""
    import torch

    from fade_b200.cache import TIER_FP16, TIER_INT2, TIER_INT4
    from fade_b200.policy import _assign_one_layer, assign_counts

    g = torch.Generator().manual_seed(0)
    for S in (0, 1, 4, 68, 69, 500, 4096):
        for n_sink, recent in ((0, 0), (4, 64)):
            for b4 in (None, 0, 1, 400, 10000):
                for b2 in (0, 10, 300):
                    t = _assign_one_layer(S, torch.rand(S, generator=g), n_sink, recent, b4, b2)
                    got = assign_counts(S, n_sink, recent, b4, b2)
                    assert got == (int((t == TIER_FP16).sum()), int((t == TIER_INT4).sum()),
                                   int((t == TIER_INT2).sum())), (S, n_sink, recent, b4, b2)
