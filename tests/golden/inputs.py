"""Seeded synthetic inputs shared by make_golden.py (which runs the reference
on them) and the GPU tests (which regenerate them on the box, where the
reference is absent).  torch's CPU generator is deterministic for a given
torch build, and every fixture also stores a checksum of the inputs it was
made from, so a test can prove it regenerated the same bits.

Shapes follow the benchmark configurations: N(0,1) with 4 outlier channels
per head scaled x8; keys RoPE'd at their positions.
"""

from __future__ import annotations

import numpy as np
import torch


def outlier_tensor(shape, gen, n_out=4, mult=8.0):
    x = torch.randn(*shape, generator=gen)
    H, D = shape[1], shape[-1]
    for h in range(H):
        ch = torch.randperm(D, generator=gen)[:n_out]
        x[:, h, :, ch] *= mult
    return x


def rope_fp32(k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """k * cos + rotate_half(k) * sin in fp32, cast back (the model's RoPE)."""
    kf = k.float()
    h = kf.shape[-1] // 2
    rot = torch.cat((-kf[..., h:], kf[..., :h]), dim=-1)
    return (kf * cos.float() + rot * sin.float()).to(k.dtype)


def checksum(t: torch.Tensor) -> int:
    """Order-sensitive checksum of a tensor's storage bits."""
    b = t.contiguous().view(torch.int16).numpy().astype(np.int64).ravel()
    w = (np.arange(b.size, dtype=np.int64) % 65521) + 1
    return int(((b & 0xFFFF) * w).sum() % (1 << 61))


# --------------------------------------------------------------- config 3
CFG3 = dict(B=1, Hq=32, Hkv=8, D=128, S=4096, n_sink=4, recent=64, budget=400, group=32, theta=1e6)


def cfg3_inputs(cos_sin):
    """Mistral-7B-shaped H2O eviction (batch sliced to 1 so the fixture stays
    small).  cos_sin(positions) -> (cos, sin) fp32 tables [1,1,S,D] of the
    Vanilla scheme (theta 1e6).  Returns k_roped, v, q (fp16) and the
    per-token scores: Dirichlet(0.1) per kv head, summed over heads."""
    c = CFG3
    gen = torch.Generator().manual_seed(31)
    k_pre = outlier_tensor((c["B"], c["Hkv"], c["S"], c["D"]), gen).to(torch.float16)
    v = outlier_tensor((c["B"], c["Hkv"], c["S"], c["D"]), gen).to(torch.float16)
    q = torch.randn(c["B"], c["Hq"], 1, c["D"], generator=gen).to(torch.float16)
    cos, sin = cos_sin(torch.arange(c["S"]))
    k = rope_fp32(k_pre, cos, sin)
    torch.manual_seed(31)
    scores = torch.distributions.Dirichlet(torch.full((c["S"],), 0.1)).sample((c["Hkv"],)).sum(0)
    return k, v, q, scores


# --------------------------------------------------------------- config 4
CFG4 = dict(Hq=28, Hkv=4, D=128, n_seq=6, lo=512, hi=4096, n_sink=4, recent=64, bits=2)


def cfg4_inputs():
    """Qwen2.5-7B-shaped ragged batch (bf16): n_seq sequences with lengths
    uniform in [lo, hi] (the benchmark's 512..32768 scaled down for the fixture).
    Returns (lengths, [(k, v) per sequence], q [n_seq, Hq, 1, D])."""
    c = CFG4
    gen = torch.Generator().manual_seed(41)
    lens = torch.randint(c["lo"], c["hi"] + 1, (c["n_seq"],), generator=gen).tolist()
    seqs = []
    for n in lens:
        k = outlier_tensor((1, c["Hkv"], n, c["D"]), gen).to(torch.bfloat16)
        v = outlier_tensor((1, c["Hkv"], n, c["D"]), gen).to(torch.bfloat16)
        seqs.append((k, v))
    q = torch.randn(c["n_seq"], c["Hq"], 1, c["D"], generator=gen).to(torch.bfloat16)
    return lens, seqs, q
