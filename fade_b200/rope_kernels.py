"""Eviction survivors: gather + un-RoPE + re-RoPE in one kernel pass.

Replaces the evicting branch of the reference's ``apply_tier_assignment``
(fade/cache.py:914-935), which un-RoPEs every cached token at its old position
(``_inverse_rope``, fade/cache.py:301-311), ``index_select``s the survivors and
re-RoPEs them at 0..n_kept-1 (``_apply_rope``, fade/cache.py:290-299).  Only
the kept rows are read; results are bit-identical given the same cos/sin
tables (the RopeScheme's, fade/rope.py:72-93).
"""

from __future__ import annotations

import torch
from torch import Tensor

from fade_b200 import _lib


def rerope_gather(k: Tensor, v: Tensor | None, keep_idx: Tensor, cos_old: Tensor | None, sin_old: Tensor | None,
                  cos_new: Tensor | None, sin_new: Tensor | None, apply_rope: bool = True):
    """k, v [B,H,S,D] -> (k_out, v_out) [B,H,n_kept,D] contiguous.

    cos/sin tables: float32 [S, D] (old positions) and [n_kept, D] (new);
    leading broadcast dims of size 1 are accepted.  With ``apply_rope=False``
    only the gather runs (NoRope models)."""
    dev = _lib.require_cuda(k, v, keep_idx)
    B, H, S, D = k.shape
    keep = keep_idx.to(device=dev, dtype=torch.int64).contiguous()
    n = keep.numel()
    k_out = torch.empty(B, H, n, D, dtype=k.dtype, device=dev)
    v_out = torch.empty(B, H, n, D, dtype=v.dtype, device=dev) if v is not None else None
    if v is not None and (v.shape != k.shape or v.stride() != k.stride()):
        v = v.contiguous()
        k = k.contiguous()

    def tab(t, rows):
        if t is None:
            return None
        t = t.to(device=dev, dtype=torch.float32).reshape(-1, D).contiguous()
        if t.shape[0] != rows:
            raise ValueError(f"cos/sin table has {t.shape[0]} rows, expected {rows}")
        return t

    co, so = tab(cos_old, S), tab(sin_old, S)
    cn, sn = tab(cos_new, n), tab(sin_new, n)
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_rerope_gather(
            k.data_ptr(), _lib.ptr(v), _lib.dtype_code(k.dtype), _lib.view4(k), keep.data_ptr(), n,
            _lib.ptr(co), _lib.ptr(so), _lib.ptr(cn), _lib.ptr(sn), 1 if apply_rope else 0,
            k_out.data_ptr(), _lib.ptr(v_out), st,
        ),
        "rerope_gather",
    )
    return k_out, v_out
