"""fade_decode_attn_noalloc: attention without a caller-supplied workspace.

Callers that cannot allocate device memory while they run (a serving runtime
working from a fixed pool, a plugin host that forbids cudaMalloc after
start-up) use this entry point; it takes its scratch space from an array built
into the library.  These tests call it through the C ABI and check it against
the workspace-based fade_decode_attn and the oracle on the same inputs, twice
in a row and with a smaller call after a larger one (the built-in array keeps
the previous call's bytes, which must not leak into the next result), read
the array's error word with fade_decode_attn_noalloc_check after each call,
and check that an oversized request is refused.

Kept in its own file, named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_attn_close, np_to_dt_tensor, seeded_outliers, t_vals
from oracle import attention as oa
from oracle import quant as oq
from oracle.numerics import rnd

pytestmark = pytest.mark.gpu


def _case(seed: int, dt: str = "bf16", B: int = 2, n_mid: int = 1500, q_nan: bool = False):
    from fade_b200.attention import FPTier, Int4Tier

    Hq, Hkv, D = 32, 8, 128
    x = seeded_outliers((B, Hkv, 4 + n_mid + 64, D), seed, dt)
    v = seeded_outliers((B, Hkv, 4 + n_mid + 64, D), seed + 1, dt)
    kp, ks = oq.quant_k_int4(x[:, :, 4:4 + n_mid], dt)
    vp, vs = oq.quant_v_int4(v[:, :, 4:4 + n_mid], dt)
    q = rnd(np.random.default_rng(seed).standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    if q_nan:
        q[:] = np.nan
    tiers = [
        FPTier(np_to_dt_tensor(x[:, :, :4], dt), np_to_dt_tensor(v[:, :, :4], dt)),
        Int4Tier(torch.from_numpy(kp).cuda(), np_to_dt_tensor(ks, dt),
                 torch.from_numpy(vp).cuda(), np_to_dt_tensor(vs, dt)),
        FPTier(np_to_dt_tensor(x[:, :, 4 + n_mid:], dt), np_to_dt_tensor(v[:, :, 4 + n_mid:], dt)),
    ]
    oracle_tiers = {"sink_k": x[:, :, :4], "sink_v": v[:, :, :4], "int4_kq": kp, "int4_ks": ks,
                    "int4_vq": vp, "int4_vs": vs, "recent_k": x[:, :, 4 + n_mid:], "recent_v": v[:, :, 4 + n_mid:]}
    return q, np_to_dt_tensor(q, dt), tiers, oracle_tiers


def _noalloc(lib, _lib, q, tiers):
    from fade_b200.attention import DecodePlan

    out = torch.full_like(q, float("nan"))
    plan = DecodePlan(q, tiers, out=out)            # descriptor only; its workspace is not used
    st = _lib.bind(q.device)
    status = lib.fade_decode_attn_noalloc(ctypes.byref(plan.desc), st)
    assert status == _lib.FADE_OK, lib.fade_status_string(status)
    # no bounded device wait gave up during the call
    assert lib.fade_decode_attn_noalloc_check(st) == _lib.FADE_OK
    return t_vals(out)


def test_noalloc_matches_workspace_entry_point(cuda_device):
    """Two calls in a row through the shared built-in array, each equal to the
    workspace-based entry point and within the attention tolerance of the
    oracle."""
    from fade_b200 import _lib
    from fade_b200.attention import DecodePlan

    lib = _lib.load()
    for seed in (11, 12):
        q_np, q, tiers, otiers = _case(seed)
        ref = t_vals(DecodePlan(q, tiers).run()).copy()   # workspace-based entry point
        out = _noalloc(lib, _lib, q, tiers)
        assert_attn_close(out, ref, "bf16", 1e-2)
        assert_attn_close(out, oa.tiered_attention(q_np, otiers, "bf16"), "bf16", 1e-2)


def test_noalloc_smaller_call_after_larger_one(cuda_device):
    """A large call whose queries are NaN leaves NaN partials all over the
    built-in array; a following call with fewer rows and fewer 128-token
    units must read none of them."""
    from fade_b200 import _lib

    lib = _lib.load()
    _, q_big, tiers_big, _ = _case(21, B=4, n_mid=3000, q_nan=True)
    big = _noalloc(lib, _lib, q_big, tiers_big)
    assert np.isnan(big).all()
    q_np, q, tiers, otiers = _case(22, B=1, n_mid=300)
    out = _noalloc(lib, _lib, q, tiers)
    assert np.isfinite(out).all()
    assert_attn_close(out, oa.tiered_attention(q_np, otiers, "bf16"), "bf16", 1e-2)


def test_noalloc_rejects_oversized_request(cuda_device):
    from fade_b200 import _lib
    from fade_b200.attention import DecodePlan

    lib = _lib.load()
    _, q, tiers, _ = _case(13)
    plan = DecodePlan(q, tiers)
    big = _lib.DecodeDesc.from_buffer_copy(plan.desc)
    big.seg[1].len = 50_000_000          # workspace far beyond the built-in array
    big.seg[1].max_len = 50_000_000
    need = lib.fade_decode_attn_workspace_size(ctypes.byref(big))
    assert need > lib.fade_decode_attn_noalloc_max_bytes()
    st = _lib.bind(q.device)
    assert lib.fade_decode_attn_noalloc(ctypes.byref(big), st) == _lib.FADE_ERR_WORKSPACE
