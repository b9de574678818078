"""The tcgen05 middle kernel (INT4 K and V at head_dim 128: dequantised K in
tensor memory, V in shared memory, S^T and O^T accumulated in tensor memory)
against the same oracle cases as the mma.sync kernel, at the same
north-star tolerances, plus a direct comparison of the two kernels."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import test_decode_gpu as td
from gpu_util import assert_attn_close, np_to_dt_tensor, t_vals

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc(cuda_device):
    from fade_b200.attention import get_middle_kernel, set_middle_kernel

    set_middle_kernel("tcgen05")
    assert get_middle_kernel() == "tcgen05"
    try:
        yield cuda_device
    finally:
        set_middle_kernel("mma_sync")


@pytest.mark.parametrize(
    "B,Hq,Hkv,D,n_sink,n_mid,n_rec,dt,n_q",
    [
        (2, 32, 8, 128, 4, 1000, 64, "bf16", 1),     # Llama-8B head shape
        (3, 8, 8, 128, 4, 129, 5, "f16", 1),         # MHA (g=1), ragged edge of a unit
        (2, 28, 4, 128, 4, 1, 64, "bf16", 1),        # a single middle token, g=7
        (1, 64, 8, 128, 4, 4096, 128, "bf16", 1),    # Llama-70B head shape
        (2, 8, 2, 128, 4, 777, 64, "f16", 3),        # 12 query rows (N = 16)
    ],
)
def test_random_vs_oracle_tc(tc, B, Hq, Hkv, D, n_sink, n_mid, n_rec, dt, n_q):
    td.test_random_vs_oracle(tc, B, Hq, Hkv, D, n_sink, n_mid, n_rec, dt, n_q)


def test_cta_counts_tc(tc):
    td.test_forced_cta_counts_agree(tc)


def test_device_lengths_and_ragged_tc(tc):
    td.test_device_lengths_and_ragged(tc)


def test_paged_int4_middle_tc(tc):
    td.test_paged_int4_middle(tc)


def test_repeat_calls_are_stable_tc(tc):
    td.test_repeat_calls_are_stable(tc)


@pytest.mark.parametrize("fused,S,cap,L", [(True, 600, 600, 2), (True, 194, 300, 1)])
def test_decoder_step_tc(tc, fused, S, cap, L):
    td.test_decoder_step_matches_oracle(tc, fused, S, cap, L)


def test_kernels_agree(cuda_device):
    """mma.sync and tcgen05 on a config-2-shaped layer: both within the
    north-star tolerance of the oracle and of each other."""
    from fade_b200.attention import set_middle_kernel, tiered_decode_attention

    q, tiers = td._random_int4_case(2, 32, 8, 128, 4, 8124, 64, "bf16", seed=77)
    qt = np_to_dt_tensor(q, "bf16")
    tt = td._torch_tiers(tiers, "bf16")
    outs = {}
    try:
        for kind in ("mma_sync", "tcgen05"):
            set_middle_kernel(kind)
            outs[kind] = t_vals(tiered_decode_attention(qt, tt))
    finally:
        set_middle_kernel("mma_sync")
    ref = td.oa.tiered_attention(q, tiers, "bf16")
    for kind, out in outs.items():
        assert_attn_close(out, ref, "bf16", td.TOL["bf16"])
    assert np.max(np.abs(outs["mma_sync"] - outs["tcgen05"])) <= 2 * td.TOL["bf16"]
