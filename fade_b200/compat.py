"""``import fade`` compatibility.

Code written against the reference package imports ``fade`` (fade-kv 1.1.0):
``from fade import FadeConfig, create_tiered_cache``,
``from fade.cache import TieredKVCache``,
``from fade.kernels.fused_int4_attn import fused_int4_sdpa`` and so on.
``install_fade_alias()`` registers this package's modules under those names,
so such code runs on the sm_100a path without edits:

    import fade_b200.compat; fade_b200.compat.install_fade_alias()
    from fade import FadeConfig, create_tiered_cache      # -> fade_b200

Only the hot-path API is aliased (config, cache, patch, backends, quant,
rotated_quant, rope, policy, fused_int4_sdpa); the reference's other
subsystems (policies beyond tier selection, server, evaluation, telemetry)
are not part of this library, and importing them raises ImportError.
"""

from __future__ import annotations

import importlib
import sys
import types

_SUBMODULES = {
    "fade.config": "fade_b200.config",
    "fade.cache": "fade_b200.cache",
    "fade.patch": "fade_b200.patch",
    "fade.backends": "fade_b200.backends",
    "fade.quant": "fade_b200.quant",
    "fade.rotated_quant": "fade_b200.rotated_quant",
    "fade.rope": "fade_b200.rope",
    "fade.policy": "fade_b200.policy",
}
_TOP = ("FadeConfig", "create_tiered_cache", "TieredKVCache", "get_backend")


def install_fade_alias(force: bool = False) -> types.ModuleType:
    """Register ``fade`` and its hot-path submodules in ``sys.modules``.
    An already imported, different ``fade`` is replaced only with ``force``."""
    cur = sys.modules.get("fade")
    if cur is not None and not getattr(cur, "__fade_b200_alias__", False) and not force:
        raise RuntimeError("another 'fade' package is already imported; pass force=True to replace it")
    top = types.ModuleType("fade", "fade_b200 under the reference's package name")
    top.__fade_b200_alias__ = True
    top.__path__ = []                      # a package: submodules resolve through sys.modules
    import fade_b200

    for name in _TOP:
        setattr(top, name, getattr(fade_b200, name))
    sys.modules["fade"] = top
    for alias, real in _SUBMODULES.items():
        mod = importlib.import_module(real)
        sys.modules[alias] = mod
        setattr(top, alias.split(".", 1)[1], mod)
    kernels = types.ModuleType("fade.kernels")
    kernels.__path__ = []
    fia = types.ModuleType("fade.kernels.fused_int4_attn")
    from fade_b200.attention import fused_int4_sdpa

    fia.fused_int4_sdpa = fused_int4_sdpa
    kernels.fused_int4_attn = fia
    top.kernels = kernels
    sys.modules["fade.kernels"] = kernels
    sys.modules["fade.kernels.fused_int4_attn"] = fia
    return top


def uninstall_fade_alias() -> None:
    """Remove the alias modules registered by install_fade_alias."""
    top = sys.modules.get("fade")
    if top is None or not getattr(top, "__fade_b200_alias__", False):
        return
    for name in [n for n in sys.modules if n == "fade" or n.startswith("fade.")]:
        del sys.modules[name]


__all__ = ["install_fade_alias", "uninstall_fade_alias"]
