"""K1 quantisers on the GPU: bit-exact against the reference's golden vectors
and the CPU oracle (codes, packed bytes and scales compared as raw bits)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import np_to_dt_tensor, seeded_outliers, t_bits, t_from_bits, t_vals
from oracle import quant as oq
from oracle import rope as orope
from oracle.numerics import from_bits, to_bits

pytestmark = pytest.mark.gpu
DTS = ("f16", "bf16")


@pytest.mark.parametrize("dt", DTS)
def test_int4_golden(cuda_device, dt):
    from fade_b200.quant import quant_k_int4, quant_v_int4

    g = golden("quant")
    x = t_from_bits(g[f"{dt}_x"], dt)
    kp, ks = quant_k_int4(x)
    vp, vs = quant_v_int4(x)
    np.testing.assert_array_equal(kp.cpu().numpy(), g[f"{dt}_k_packed"])
    np.testing.assert_array_equal(t_bits(ks), g[f"{dt}_k_scale"])
    np.testing.assert_array_equal(vp.cpu().numpy(), g[f"{dt}_v_packed"])
    np.testing.assert_array_equal(t_bits(vs), g[f"{dt}_v_scale"])


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("G", (32, 64))
def test_int2_golden(cuda_device, dt, G):
    from fade_b200.quant import quant_int2_grouped_packed, quant_k_int2, quant_v_int2

    g = golden("quant")
    x = t_from_bits(g[f"{dt}_x2"], dt)
    kq, ks = quant_k_int2(x, group_size=G)
    vq, vs = quant_v_int2(x, group_size=G)
    np.testing.assert_array_equal(kq.cpu().numpy(), g[f"{dt}_k2_g{G}_codes"])
    np.testing.assert_array_equal(t_bits(ks), g[f"{dt}_k2_g{G}_scale"])
    np.testing.assert_array_equal(vq.cpu().numpy(), g[f"{dt}_v2_g{G}_codes"])
    np.testing.assert_array_equal(t_bits(vs), g[f"{dt}_v2_g{G}_scale"])
    qp, sp = quant_int2_grouped_packed(x, G)
    np.testing.assert_array_equal(qp.cpu().numpy(), oq.pack2(g[f"{dt}_v2_g{G}_codes"]))
    np.testing.assert_array_equal(t_bits(sp), g[f"{dt}_v2_g{G}_scale"])


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("shape", [(2, 4, 1000, 128), (1, 2, 2048, 64), (3, 1, 7, 96), (1, 1, 1, 6),
                                   (1, 3, 1337, 256), (2, 2, 513, 128)])
def test_int4_vs_oracle_random(cuda_device, dt, shape):
    from fade_b200.quant import quant_k_int4, quant_v_int4

    x = seeded_outliers(shape, seed=sum(shape), dt=dt)
    xt = np_to_dt_tensor(x, dt)
    kp, ks = quant_k_int4(xt)
    vp, vs = quant_v_int4(xt)
    okp, oks = oq.quant_k_int4(x, dt)
    ovp, ovs = oq.quant_v_int4(x, dt)
    np.testing.assert_array_equal(kp.cpu().numpy(), okp)
    np.testing.assert_array_equal(t_bits(ks), to_bits(oks, dt))
    np.testing.assert_array_equal(vp.cpu().numpy(), ovp)
    np.testing.assert_array_equal(t_bits(vs), to_bits(ovs, dt))


def test_int4_strided_input(cuda_device):
    """Non-contiguous views (e.g. an index_select-free slice of a bigger cache)."""
    from fade_b200.quant import quant_k_int4, quant_v_int4

    x = seeded_outliers((2, 3, 2100, 128), seed=5, dt="f16")
    big = np_to_dt_tensor(x, "f16")
    # short rows (one CTA per (b, h) channel block), longer rows (clusters per (b, h))
    for lo, hi in ((17, 250), (17, 800), (17, 2090)):
        view = big[:, :, lo:hi]          # strided along S (still contiguous rows)
        tview = big.transpose(1, 2).contiguous().transpose(1, 2)[:, :, lo:hi]  # exotic strides
        okp, oks = oq.quant_k_int4(x[:, :, lo:hi], "f16")
        ovp, ovs = oq.quant_v_int4(x[:, :, lo:hi], "f16")
        for t in (view, tview):
            kp, ks = quant_k_int4(t)
            vp, vs = quant_v_int4(t)
            np.testing.assert_array_equal(kp.cpu().numpy(), okp)
            np.testing.assert_array_equal(t_bits(ks), to_bits(oks, "f16"))
            np.testing.assert_array_equal(vp.cpu().numpy(), ovp)
            np.testing.assert_array_equal(t_bits(vs), to_bits(ovs, "f16"))


def test_errors_match_reference_messages(cuda_device):
    from fade_b200.quant import _pack_int4_last_dim, quant_k_int2, quant_k_int4

    x = torch.zeros(1, 1, 4, 3, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="last dim must be even for INT4 packing, got 3"):
        quant_k_int4(x)
    with pytest.raises(ValueError, match="last dim must be even for INT4 packing"):
        _pack_int4_last_dim(torch.zeros(2, 5, dtype=torch.int8, device="cuda"))
    with pytest.raises(ValueError, match="S=10 must be divisible by group_size=4"):
        quant_k_int2(torch.zeros(1, 1, 10, 8, dtype=torch.float16, device="cuda"), group_size=4)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        quant_k_int4(torch.zeros(1, 1, 4, 4, dtype=torch.float16))


def test_zero_and_nan_edge_cases(cuda_device):
    """fp16 all-zero channel -> scale 0 and code 0 (0*inf = NaN -> 0), like torch on CPU."""
    from fade_b200.quant import quant_k_int4, quant_v_int4

    x = torch.zeros(1, 2, 5, 8, dtype=torch.float16, device="cuda")
    kp, ks = quant_k_int4(x)
    vp, vs = quant_v_int4(x)
    assert int(kp.abs().sum()) == 0 and float(ks.abs().sum()) == 0.0
    assert int(vp.abs().sum()) == 0 and float(vs.abs().sum()) == 0.0


@pytest.mark.parametrize("dt", DTS)
def test_pack_unpack_dequant(cuda_device, dt):
    from fade_b200.quant import (_pack_int2_last_dim, _pack_int4_last_dim, _unpack_int2_last_dim,
                                 _unpack_int4_last_dim, dequant_int2_packed, dequant_int4,
                                 dequant_v_int2, quant_k_int4, quant_v_int2, quant_v_int4)

    rng = np.random.default_rng(3)
    q4 = torch.from_numpy(rng.integers(-8, 8, size=(2, 3, 33, 64)).astype(np.int8)).cuda()
    p4 = _pack_int4_last_dim(q4)
    np.testing.assert_array_equal(p4.cpu().numpy(), oq.pack_int4(q4.cpu().numpy()))
    assert torch.equal(_unpack_int4_last_dim(p4), q4)
    q2 = torch.from_numpy(rng.integers(-2, 2, size=(2, 3, 33, 64)).astype(np.int8)).cuda()
    p2 = _pack_int2_last_dim(q2)
    np.testing.assert_array_equal(p2.cpu().numpy(), oq.pack2(q2.cpu().numpy()))
    assert torch.equal(_unpack_int2_last_dim(p2), q2)

    x = seeded_outliers((2, 3, 64, 64), seed=9, dt=dt)
    xt = np_to_dt_tensor(x, dt)
    kp, ks = quant_k_int4(xt)
    vp, vs = quant_v_int4(xt)
    okp, oks = oq.quant_k_int4(x, dt)
    ovp, ovs = oq.quant_v_int4(x, dt)
    np.testing.assert_array_equal(t_bits(dequant_int4(kp, ks, dtype=xt.dtype)), to_bits(oq.dequant_int4(okp, oks, dt), dt))
    np.testing.assert_array_equal(t_bits(dequant_int4(vp, vs, dtype=xt.dtype)), to_bits(oq.dequant_int4(ovp, ovs, dt), dt))
    q, s = quant_v_int2(xt, group_size=32)
    oqq, oss = oq.quant_int2_grouped(x, 32, dt)
    ref = to_bits(oq.dequant_grouped(oqq, oss, 32, dt), dt)
    np.testing.assert_array_equal(t_bits(dequant_v_int2(q, s, group_size=32, dtype=xt.dtype)), ref)
    np.testing.assert_array_equal(t_bits(dequant_int2_packed(_pack_int2_last_dim(q), s, 32, dtype=xt.dtype)), ref)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("D", (64, 128))
@pytest.mark.parametrize("bits", (2, 4))
def test_rotated_quant(cuda_device, dt, D, bits):
    """CUDA-core path (f16, D = 64): bit-exact vs the oracle (same sequential
    fp32 order).  Tensor-core path (bf16 at D = 128): the rotation sums exact
    products in the tensor core's order, so against the oracle codes may
    differ by one where a rotated value sits within fp32 rounding of a
    boundary and scales by one ulp; the dequantisation of its own codes is
    bit-exact.  Against the reference (its own matmul order) both paths are
    within one code on < 0.2 % of entries."""
    from fade_b200 import _lib
    from fade_b200.rotated_quant import rotated_dequant_k, rotated_dequant_v, rotated_quant_k, rotated_quant_v

    g = golden("rotated")
    R = g[f"R{D}"]
    Rt = torch.from_numpy(R).cuda()
    xb = g[f"{dt}_D{D}_x"]
    x = from_bits(xb, dt)
    xt = t_from_bits(xb, dt)
    tensor_cores = dt == "bf16" and D == 128
    unpack = oq.unpack_int4 if bits == 4 else oq.unpack2
    for kind, qf, dqf in (("k", rotated_quant_k, rotated_dequant_k), ("v", rotated_quant_v, rotated_dequant_v)):
        p, s = qf(xt, Rt, bits=bits)
        assert _lib.load().fade_rotated_quant_check(_lib.bind(xt.device)) == 0
        op, os_ = oq.rotated_quant(x, R, bits, kind, dt)
        if tensor_cores:
            assert_rot_close(p.cpu().numpy(), s, op, os_, unpack, dt)
            gp, gs = p.cpu().numpy(), from_bits(t_bits(s), dt)
        else:
            np.testing.assert_array_equal(p.cpu().numpy(), op)
            np.testing.assert_array_equal(t_bits(s), to_bits(os_, dt))
            gp, gs = op, os_
        deq = dqf(p, s, Rt, bits=bits, dtype=xt.dtype)
        np.testing.assert_array_equal(t_bits(deq), to_bits(oq.rotated_dequant(gp, gs, R, bits, dt), dt))
        diff = np.abs(unpack(p.cpu().numpy()).astype(int) - unpack(g[f"{dt}_D{D}_b{bits}_{kind}_packed"]).astype(int))
        assert diff.max() <= 1 and (diff != 0).mean() < 2e-3


def assert_rot_close(p, s, op, os_, unpack, dt, frac=1e-3):
    """Tensor-core rotated quantisation vs the oracle: codes within one on at
    most `frac` of the entries, scales within one ulp of the dtype."""
    d = np.abs(unpack(p).astype(int) - unpack(op).astype(int))
    assert d.max() <= 1 and (d != 0).mean() <= frac, (d.max(), (d != 0).mean())
    sb = t_bits(s).astype(np.int64)
    ob = to_bits(os_, dt).astype(np.int64)
    assert np.abs(sb - ob).max() <= 1
    print(f"[rotated tc] codes differing from the oracle: {(d != 0).mean():.2e}, "
          f"scales differing: {(sb != ob).mean():.2e}")


@pytest.mark.parametrize("bits", (2, 4))
def test_rotated_quant_tensor_core_tiles(cuda_device, bits):
    """bf16 tensor-core rotation over many 128-token tiles (partial last tile,
    several (b, h) rows, a strided view): codes and scales against the oracle,
    and the dequantisation of its own codes bit-exact."""
    from fade_b200 import _lib
    from fade_b200.rotated_quant import _random_orthogonal, rotated_dequant_k, rotated_dequant_v, rotated_quant_k, \
        rotated_quant_v

    dt = "bf16"
    R = _random_orthogonal(128, 3).numpy().astype(np.float32)
    Rt = torch.from_numpy(R).cuda()
    xs = seeded_outliers((2, 3, 700, 128), 91, dt)
    xt_full = np_to_dt_tensor(xs, dt)
    for xt in (xt_full, xt_full[:, :, 50:650]):   # contiguous, then a view with a row offset
        x = xt.float().cpu().numpy()
        unpack = oq.unpack_int4 if bits == 4 else oq.unpack2
        for kind, qf, dqf in (("k", rotated_quant_k, rotated_dequant_k), ("v", rotated_quant_v, rotated_dequant_v)):
            p, s = qf(xt, Rt, bits=bits)
            assert _lib.load().fade_rotated_quant_check(_lib.bind(xt.device)) == 0
            op, os_ = oq.rotated_quant(x, R, bits, kind, dt)
            assert_rot_close(p.cpu().numpy(), s, op, os_, unpack, dt)
            deq = dqf(p, s, Rt, bits=bits, dtype=xt.dtype)
            ref = oq.rotated_dequant(p.cpu().numpy(), from_bits(t_bits(s), dt), R, bits, dt)
            np.testing.assert_array_equal(t_bits(deq), to_bits(ref, dt))


@pytest.mark.parametrize("dt", DTS)
def test_rerope_golden(cuda_device, dt):
    from fade_b200.rope_kernels import rerope_gather

    g = golden("rope")
    k = t_from_bits(g[f"{dt}_k"], dt)
    keep = torch.from_numpy(g[f"{dt}_keep"]).cuda()
    tabs = [torch.from_numpy(g[f"{dt}_{n}"]).cuda() for n in ("cos_old", "sin_old", "cos_new", "sin_new")]
    v = torch.randn_like(k.float()).to(k.dtype)
    ko, vo = rerope_gather(k, v, keep, *tabs)
    np.testing.assert_array_equal(t_bits(ko), g[f"{dt}_out"])
    assert torch.equal(vo, v.index_select(2, keep))


@pytest.mark.parametrize("dt", DTS)
def test_rerope_vs_oracle_large(cuda_device, dt):
    from fade_b200.rope_kernels import rerope_gather

    B, H, S, D = 2, 8, 4096, 128
    x = seeded_outliers((B, H, S, D), seed=11, dt=dt)
    rng = np.random.default_rng(1)
    keep = np.sort(rng.choice(S, size=468, replace=False))
    co, so = orope.vanilla_cos_sin(np.arange(S), D, 1e6, dt)
    cn, sn = orope.vanilla_cos_sin(np.arange(468), D, 1e6, dt)
    ref = orope.rerope_gather(x, keep, co, so, cn, sn, dt)
    xt = np_to_dt_tensor(x, dt)
    tabs = [torch.from_numpy(a).cuda() for a in (co, so, cn, sn)]
    ko, _ = rerope_gather(xt, None, torch.from_numpy(keep).cuda(), *tabs)
    np.testing.assert_array_equal(t_bits(ko), to_bits(ref, dt))


@pytest.mark.parametrize("dt", DTS)
def test_age_out_vs_oracle(cuda_device, dt):
    from fade_b200.decoder import age_out_int4

    B, H, D, R, cap = 3, 4, 128, 8, 40
    rng = np.random.default_rng(7)
    ring = seeded_outliers((B, H, R, D), seed=1, dt=dt)
    ringv = seeded_outliers((B, H, R, D), seed=2, dt=dt)
    ks = np.abs(seeded_outliers((B, H, 1, D), seed=3, dt=dt))[:, :, 0] / 7
    ks = from_bits(to_bits(ks, dt), dt)
    ks[0, 0, 3] = 0.0
    new_k = seeded_outliers((B, H, 1, D), seed=4, dt=dt)[:, :, 0]
    new_v = seeded_outliers((B, H, 1, D), seed=5, dt=dt)[:, :, 0]
    n0 = np.array([5, 9, 0], dtype=np.int32)
    origin = 2
    rk, rv = np_to_dt_tensor(ring, dt), np_to_dt_tensor(ringv, dt)
    kpk = torch.zeros(B, H, cap, D // 2, dtype=torch.uint8, device="cuda")
    vpk = torch.zeros_like(kpk)
    vsc = torch.zeros(B, H, cap, 1, dtype=rk.dtype, device="cuda")
    mid_len = torch.from_numpy(n0.copy()).cuda()
    age_out_int4(rk, rv, kpk, vpk, vsc, np_to_dt_tensor(ks, dt), mid_len, ring_origin=origin,
                 k_new=np_to_dt_tensor(new_k, dt), v_new=np_to_dt_tensor(new_v, dt))
    assert mid_len.cpu().tolist() == [6, 10, 1]
    for b in range(B):
        slot = (n0[b] - origin) % R
        okp, ovp, ovs = oq.age_out_int4(ring[b, :, slot], ringv[b, :, slot], ks[b], dt)
        np.testing.assert_array_equal(kpk[b, :, n0[b]].cpu().numpy(), okp)
        np.testing.assert_array_equal(vpk[b, :, n0[b]].cpu().numpy(), ovp)
        np.testing.assert_array_equal(t_bits(vsc[b, :, n0[b], 0]), to_bits(ovs, dt))
        np.testing.assert_array_equal(t_vals(rk[b, :, slot]), new_k[b])
        np.testing.assert_array_equal(t_vals(rv[b, :, slot]), new_v[b])
