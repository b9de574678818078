"""Model integration (the reference's ``fade/patch.py:125-207``).

``create_tiered_cache(model, dtype, config=None, **kwargs)`` builds a
``TieredKVCache`` from the model's RoPE parameters and head_dim, as the
reference does (recurrent models get a plain DynamicCache, MLA models and
linear-attention layers are passed through).  In addition it binds the cache
to the model's attention modules and registers the ``"fade_tiered"``
attention implementation: on single-token decode steps that function runs
the fused tiered decode kernel over the cache's compressed tiers
(``TieredKVCache.decode_attention``); prefill, masked batches and unmanaged
layers take transformers' SDPA path on the materialised cache.  Pass
``fused_attention=False`` to leave the model's attention untouched.
"""

from __future__ import annotations

import warnings
import weakref

import torch
from transformers.cache_utils import DynamicCache

from fade_b200.cache import TieredKVCache
from fade_b200.config import FadeConfig
from fade_b200.rope import extract_rope_scheme

ATTN_IMPL = "fade_tiered"
_RECURRENT = {"mamba", "mamba2", "rwkv", "rwkv5", "rwkv6", "xlstm"}
_MLA = {"deepseek", "deepseek_r1", "deepseek_r2", "deepseek_v2", "deepseek_v3"}


def _sdpa(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kwargs):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


def fade_tiered_attention(module, query, key, value, attention_mask, dropout: float = 0.0,
                          scaling: float | None = None, is_causal: bool | None = None, **kwargs):
    """Attention function for ``attn_implementation="fade_tiered"``:
    query [B, Hq, q, D] -> (out [B, q, Hq, D], None)."""
    ref = getattr(module, "_fade_cache", None)
    cache = ref() if ref is not None else None
    layer = getattr(module, "layer_idx", None)
    fused = (cache is not None and cache.fused_decode and layer is not None and cache.is_managed(layer)
             and query.shape[2] == 1 and attention_mask is None and dropout == 0.0)
    if fused:
        out = cache.decode_attention(layer, query, scaling=scaling)
        return out.transpose(1, 2).contiguous(), None
    if cache is not None and cache.fused_decode and layer is not None and cache.is_managed(layer) \
            and query.shape[2] == 1:
        # update() returned only the new token: attend over the whole cache
        key, value = cache._materialize(layer)
    return _sdpa(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                 is_causal=is_causal, **kwargs)


def register_fade_attention() -> str:
    """Register ``"fade_tiered"`` with transformers' attention interface
    (idempotent) and return the name."""
    from transformers import AttentionInterface

    AttentionInterface.register(ATTN_IMPL, fade_tiered_attention)
    try:   # masks: same as SDPA (None when no padding, so decode stays fused)
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask

        ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_IMPL, sdpa_mask)
    except Exception:  # pragma: no cover - older transformers
        pass
    return ATTN_IMPL


def _bind(model, cache: TieredKVCache) -> None:
    n = 0
    for mod in model.modules():
        if hasattr(mod, "layer_idx") and hasattr(mod, "num_key_value_groups"):
            mod._fade_cache = weakref.ref(cache)
            n += 1
    if n == 0:
        warnings.warn("no attention modules with layer_idx found; fused decode disabled", RuntimeWarning,
                      stacklevel=3)
        return
    register_fade_attention()
    cfg = model.config
    try:
        model.set_attn_implementation(ATTN_IMPL)
    except Exception:
        cfg._attn_implementation = ATTN_IMPL
        text = getattr(cfg, "text_config", None)
        if text is not None:
            text._attn_implementation = ATTN_IMPL
    cache.fused_decode = True


def create_tiered_cache(model, dtype: torch.dtype = torch.float16, config: FadeConfig | None = None,
                        fused_attention: bool = True, **kwargs) -> TieredKVCache:
    """A ``TieredKVCache`` configured from the model (RoPE scheme, head_dim,
    skipped layers); ``config`` supplies cache knobs, ``kwargs`` override
    them.  With ``fused_attention`` the model's decode attention runs the
    fused tiered kernel over this cache."""
    cfg = model.config
    text = getattr(cfg, "text_config", cfg)
    model_type = getattr(text, "model_type", "")
    if model_type in _RECURRENT:
        warnings.warn(
            f"Model type {model_type!r} is a recurrent architecture with no standard K/V cache. "
            "Returning a plain DynamicCache. FADE tier compression is not applicable.",
            RuntimeWarning, stacklevel=2)
        return DynamicCache()  # type: ignore[return-value]
    head_dim = getattr(text, "head_dim", None) or text.hidden_size // text.num_attention_heads
    scheme = extract_rope_scheme(text, head_dim=head_dim)
    ck: dict = dict(config.to_cache_kwargs()) if config is not None else {}
    ck.update(kwargs)
    cache = TieredKVCache(dtype=dtype, rope_theta=scheme.theta, head_dim=head_dim, rope_scheme=scheme, **ck)
    layer_types = getattr(text, "layer_types", None)
    if layer_types is not None:
        skip = {i for i, lt in enumerate(layer_types) if lt not in ("full_attention", "sliding_attention")}
        if skip:
            cache.set_skip_layers(skip)
    if model_type in _MLA:
        warnings.warn(
            f"Model type {model_type!r} uses Multi-head Latent Attention. K/V are already compressed latent "
            "vectors. FADE tier management is disabled (all layers skipped). The cache still works as a "
            "DynamicCache for normal inference.", RuntimeWarning, stacklevel=2)
        cache.set_skip_layers(set(range(getattr(text, "num_hidden_layers", 0))))
        fused_attention = False
    if fused_attention:
        _bind(model, cache)
    return cache


__all__ = ["ATTN_IMPL", "create_tiered_cache", "fade_tiered_attention", "register_fade_attention"]
