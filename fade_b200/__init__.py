"""fade_b200: FADE's tiered KV-cache decode path, rebuilt for B200 (sm_100a).

The public API mirrors the reference package ``fade`` (fade-kv 1.1.0):
``FadeConfig``, ``create_tiered_cache``, ``TieredKVCache``, ``get_backend`` and
the quantisers in ``fade_b200.quant`` / ``fade_b200.rotated_quant``.  Compute
runs in ``libfade_sm100.so`` (hand-written CUDA for sm_100a behind a C ABI);
there is no CPU fallback.
"""

from __future__ import annotations

__version__ = "0.1.0"

_LAZY = {
    "FadeConfig": ("fade_b200.config", "FadeConfig"),
    "TieredKVCache": ("fade_b200.cache", "TieredKVCache"),
    "create_tiered_cache": ("fade_b200.patch", "create_tiered_cache"),
    "get_backend": ("fade_b200.backends", "get_backend"),
    "tiered_decode_attention": ("fade_b200.attention", "tiered_decode_attention"),
    "fused_int4_sdpa": ("fade_b200.attention", "fused_int4_sdpa"),
    "TieredDecoder": ("fade_b200.decoder", "TieredDecoder"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(mod), attr)
    raise AttributeError(name)


__all__ = list(_LAZY)
