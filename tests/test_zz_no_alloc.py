"""fade_decode_attn_noalloc: attention without a caller-supplied workspace.

Callers that cannot allocate device memory while they run (a serving runtime
working from a fixed pool, a plugin host that forbids cudaMalloc after
start-up) use this entry point; it takes its scratch space from an array built
into the library.  This test calls it through the C ABI and checks it against
the workspace-based fade_decode_attn on the same inputs, twice in a row (the
built-in array keeps the previous call's bytes, which must not leak into the
next result), and checks that an oversized request is refused.

Kept in its own file, named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_attn_close, np_to_dt_tensor, seeded_outliers, t_vals
from oracle import quant as oq
from oracle.numerics import rnd

pytestmark = pytest.mark.gpu


def _case(seed: int, dt: str = "bf16"):
    from fade_b200.attention import FPTier, Int4Tier

    B, Hq, Hkv, D, n_mid = 2, 32, 8, 128, 1500
    x = seeded_outliers((B, Hkv, 4 + n_mid + 64, D), seed, dt)
    v = seeded_outliers((B, Hkv, 4 + n_mid + 64, D), seed + 1, dt)
    kp, ks = oq.quant_k_int4(x[:, :, 4:4 + n_mid], dt)
    vp, vs = oq.quant_v_int4(v[:, :, 4:4 + n_mid], dt)
    q = rnd(np.random.default_rng(seed).standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    tiers = [
        FPTier(np_to_dt_tensor(x[:, :, :4], dt), np_to_dt_tensor(v[:, :, :4], dt)),
        Int4Tier(torch.from_numpy(kp).cuda(), np_to_dt_tensor(ks, dt),
                 torch.from_numpy(vp).cuda(), np_to_dt_tensor(vs, dt)),
        FPTier(np_to_dt_tensor(x[:, :, 4 + n_mid:], dt), np_to_dt_tensor(v[:, :, 4 + n_mid:], dt)),
    ]
    return np_to_dt_tensor(q, dt), tiers


def test_noalloc_matches_workspace_entry_point(cuda_device):
    from fade_b200 import _lib
    from fade_b200.attention import DecodePlan

    lib = _lib.load()
    for seed in (11, 12):  # two calls in a row through the shared built-in array
        q, tiers = _case(seed)
        ref_plan = DecodePlan(q, tiers)                 # workspace-based entry point
        ref = t_vals(ref_plan.run()).copy()
        out = torch.full_like(q, float("nan"))
        plan = DecodePlan(q, tiers, out=out)            # same descriptor, our own output
        st = _lib.bind(q.device)
        status = lib.fade_decode_attn_noalloc(ctypes.byref(plan.desc), st)
        assert status == _lib.FADE_OK, lib.fade_status_string(status)
        torch.cuda.synchronize()
        assert_attn_close(t_vals(out), ref, "bf16", 1e-2)


def test_noalloc_rejects_oversized_request(cuda_device):
    from fade_b200 import _lib
    from fade_b200.attention import DecodePlan

    lib = _lib.load()
    q, tiers = _case(13)
    plan = DecodePlan(q, tiers)
    big = _lib.DecodeDesc.from_buffer_copy(plan.desc)
    big.seg[1].len = 50_000_000          # workspace far beyond the built-in array
    big.seg[1].max_len = 50_000_000
    need = lib.fade_decode_attn_workspace_size(ctypes.byref(big))
    assert need > lib.fade_decode_attn_noalloc_max_bytes()
    st = _lib.bind(q.device)
    assert lib.fade_decode_attn_noalloc(ctypes.byref(big), st) == _lib.FADE_ERR_WORKSPACE
