"""Fused tiered decode attention (host side of ``fade_decode_attn``).

One call computes, for every (batch row, query head), softmax attention of the
decode query over the union of the cache tiers -- FP16/BF16 sink and recent
tokens plus an INT4 / INT4K-INT2V / rotated 2-or-4-bit middle -- reading the
compressed tiers straight from HBM.  It replaces the reference's per-step
``_materialize`` (fade/cache.py:693-808) + SDPA (transformers
sdpa_attention.py:40-62) and its standalone ``fused_int4_sdpa``
(fade/kernels/fused_int4_attn.py:277-342).

Tier tensors use the cache's own layouts ([B, Hkv, S, row] with contiguous
rows); views into larger capacity buffers are fine.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
from torch import Tensor

from fade_b200 import _lib


@dataclass
class FPTier:
    """Unquantised tier (sink or recent window): k, v [B, Hkv, L, D] in the model dtype."""

    k: Tensor
    v: Tensor
    lens: Tensor | None = None      # optional device int32 [B] (ragged lengths)


@dataclass
class Int4Tier:
    """INT4 middle: K per-channel (k_scale [B,Hkv,1,D]), V per-token (v_scale [B,Hkv,S,1]).

    Paged form: with ``page_table`` (int32 [B*Hkv, pages_per_row] on the
    device), k_packed / v_packed are a page pool [n_pages*128, D/2] and
    v_scale [n_pages*128, 1]; token t of (b, h) lives at pool row
    ``page_table[b*Hkv + h, t // 128] * 128 + t % 128``.  ``lens`` / ``max_len``
    give the tokens per batch row (``max_len`` defaults to the table's capacity)."""

    k_packed: Tensor
    k_scale: Tensor
    v_packed: Tensor
    v_scale: Tensor
    lens: Tensor | None = None
    max_len: int | None = None
    page_table: Tensor | None = None


@dataclass
class Int4K2VTier:
    """INT4 K (per-channel) + grouped 2-bit V (v_packed [B,Hkv,S_pad,D/4], v_scale [B,Hkv,S_pad/G,D])."""

    k_packed: Tensor
    k_scale: Tensor
    v_packed: Tensor
    v_scale: Tensor
    group: int
    length: int | None = None       # valid tokens (<= S_pad)
    lens: Tensor | None = None
    max_len: int | None = None


@dataclass
class RotTier:
    """Rotated middle (fade/rotated_quant.py): codes at `bits`, K per-channel, V per-token."""

    k_packed: Tensor
    k_scale: Tensor
    v_packed: Tensor
    v_scale: Tensor
    bits: int
    rotation: Tensor                # [D, D] float32 on the device
    lens: Tensor | None = None
    max_len: int | None = None


def _row_strides(t: Tensor, row: int, what: str) -> tuple[int, int]:
    if t.dim() != 4 or t.stride(3) != 1 or t.stride(2) != row:
        raise ValueError(f"{what}: rows of {row} elements must be contiguous, got strides {t.stride()}")
    sb, sh = t.stride(0), t.stride(1)
    if sb % row or sh % row:
        raise ValueError(f"{what}: batch/head strides must be whole rows, got {t.stride()}")
    return sb // row, sh // row


def _rows_available(t: Tensor, row_elems: int) -> int:
    """Rows addressable from t.data_ptr() to the end of its storage."""
    nbytes = t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()
    return nbytes // (row_elems * t.element_size())


def _fill_fp(seg: _lib.KVSegment, tier: FPTier, D: int) -> list:
    seg.kind = _lib.SEG_FP
    sb, sh = _row_strides(tier.k, D, "fp tier k")
    if _row_strides(tier.v, D, "fp tier v") != (sb, sh):
        raise ValueError("fp tier k and v must share a layout")
    seg.k, seg.v = tier.k.data_ptr(), tier.v.data_ptr()
    seg.row_sb, seg.row_sh = sb, sh
    L = tier.k.shape[2]
    seg.len = L
    seg.max_len = L
    if tier.lens is not None:
        seg.lens = tier.lens.data_ptr()
    return [tier.k, tier.v, tier.lens]


def _pad_rows(t: Tensor, S_pad: int) -> Tensor:
    B, H, S = t.shape[:3]
    out = torch.zeros((B, H, S_pad) + tuple(t.shape[3:]), dtype=t.dtype, device=t.device)
    out[:, :, :S] = t
    return out


def _row_aligned(tier, rbk: int, rbv: int) -> bool:
    """The middle kernel streams codes as 128-byte rows: every (b, h) segment must
    start on one and the arrays must end on one."""
    tpr = 128 // min(rbk, rbv)
    for t, rb in ((tier.k_packed, rbk), (tier.v_packed, rbv)):
        if t.stride(-1) != 1 or t.stride(2) != rb or t.stride(0) % (rb * tpr) or t.stride(1) % (rb * tpr):
            return False
        if t.storage_offset() % 128 or (_rows_available(t, rb) * rb) % 128:
            return False
    return True


def _code_bits(tier) -> tuple[int, int]:
    if isinstance(tier, Int4Tier):
        return 4, 4
    if isinstance(tier, Int4K2VTier):
        return 4, 2
    if isinstance(tier, RotTier):
        return tier.bits, tier.bits
    raise TypeError(f"unknown tier {type(tier)}")


def align_tier(tier, D: int):
    """A copy of a quantised tier that the middle kernel can stream: each
    (b, h) segment padded to a multiple of 128 tokens so it starts on a
    128-byte code row (the tier itself when it already does).  Caches that
    keep a tier across many decode steps align it once."""
    import dataclasses

    kb, vb = _code_bits(tier)
    same_rows = tier.k_packed.shape[2] == tier.v_packed.shape[2]
    if tier.lens is not None or (same_rows and _row_aligned(tier, D * kb // 8, D * vb // 8)):
        return tier
    S = tier.k_packed.shape[2]          # valid tokens (V may carry group padding beyond)
    S_pad = -(-max(S, tier.v_packed.shape[2]) // 128) * 128
    changes = dict(k_packed=_pad_rows(tier.k_packed, S_pad), v_packed=_pad_rows(tier.v_packed, S_pad))
    if isinstance(tier, Int4K2VTier):
        G = int(tier.group)
        changes["v_scale"] = _pad_rows(tier.v_scale, S_pad // G)
        changes["length"] = tier.length if tier.length is not None else S
    else:
        changes["v_scale"] = _pad_rows(tier.v_scale, S_pad)
        changes["max_len"] = tier.max_len if tier.max_len is not None else S
    return dataclasses.replace(tier, **changes)


def _fill_paged(seg: _lib.KVSegment, tier: Int4Tier, D: int, dtype: torch.dtype) -> list:
    """A paged INT4 middle: page pool + block table (see Int4Tier)."""
    seg.kind = _lib.SEG_INT4
    rb = D // 2
    kp, vp, vs, pt = tier.k_packed, tier.v_packed, tier.v_scale, tier.page_table
    if kp.dim() != 2 or kp.shape[1] != rb or not kp.is_contiguous() or vp.shape != kp.shape or not vp.is_contiguous():
        raise ValueError("paged middle: k_packed / v_packed must be contiguous pools [n_pages*128, D/2]")
    rows = int(kp.shape[0])
    if rows % _lib.PAGE_TOKENS or kp.storage_offset() % 128 or vp.storage_offset() % 128:
        raise ValueError("paged middle: pools must hold whole 128-token pages and start 128-byte aligned")
    if vs.dtype != dtype or vs.numel() != rows or not vs.is_contiguous():
        raise ValueError("paged middle: v_scale must be a contiguous [n_pages*128, 1] pool in the model dtype")
    if pt.dtype != torch.int32 or pt.dim() != 2 or not pt.is_contiguous():
        raise ValueError("page_table must be a contiguous int32 [B*Hkv, pages_per_row] tensor")
    ks = tier.k_scale
    if ks.dtype != dtype or ks.stride(-1) != 1:
        raise ValueError("k_scale must be contiguous in D and in the model dtype")
    seg.k, seg.v = kp.data_ptr(), vp.data_ptr()
    seg.row_sb = seg.row_sh = 0
    seg.k_scale, seg.ks_sb, seg.ks_sh = ks.data_ptr(), ks.stride(0), ks.stride(1)
    seg.v_scale = vs.data_ptr()
    seg.page_table, seg.pages_per_row = pt.data_ptr(), int(pt.shape[1])
    cap = int(pt.shape[1]) * _lib.PAGE_TOKENS
    seg.max_len = int(tier.max_len) if tier.max_len is not None else cap
    seg.len = seg.max_len
    if tier.lens is not None:
        seg.lens = tier.lens.data_ptr()
    seg.n_rows = rows
    return [kp, vp, ks, vs, pt, tier.lens]


def _fill_mid(seg: _lib.KVSegment, tier, D: int, dtype: torch.dtype) -> list:
    if isinstance(tier, Int4Tier) and tier.page_table is not None:
        return _fill_paged(seg, tier, D, dtype)
    if isinstance(tier, Int4Tier):
        seg.kind, kb, vb = _lib.SEG_INT4, 4, 4
    elif isinstance(tier, Int4K2VTier):
        seg.kind, kb, vb = _lib.SEG_INT4K_INT2V, 4, 2
        seg.group = int(tier.group)
    elif isinstance(tier, RotTier):
        seg.kind, kb, vb = _lib.SEG_ROT, tier.bits, tier.bits
        seg.bits = int(tier.bits)
    else:
        raise TypeError(f"unknown tier {type(tier)}")
    rbk, rbv = D * kb // 8, D * vb // 8
    if tier.lens is None and (not _row_aligned(tier, rbk, rbv)
                              or tier.k_packed.shape[2] != tier.v_packed.shape[2]):
        tier = align_tier(tier, D)
        if isinstance(tier, (Int4Tier, RotTier)):
            seg.len = tier.max_len
    sb, sh = _row_strides(tier.k_packed, rbk, "middle k codes")
    if _row_strides(tier.v_packed, rbv, "middle v codes") != (sb, sh):
        raise ValueError("middle K and V codes must share a row layout")
    seg.k, seg.v = tier.k_packed.data_ptr(), tier.v_packed.data_ptr()
    seg.row_sb, seg.row_sh = sb, sh
    ks = tier.k_scale
    if ks.dtype != dtype or ks.stride(-1) != 1:
        raise ValueError("k_scale must be contiguous in D and in the model dtype")
    seg.k_scale = ks.data_ptr()
    seg.ks_sb, seg.ks_sh = ks.stride(0), ks.stride(1)
    vs = tier.v_scale
    if vs.dtype != dtype:
        raise ValueError("v_scale must be in the model dtype")
    if isinstance(tier, Int4K2VTier):
        G = int(tier.group)
        if vs.stride(3) != 1 or vs.stride(2) != D or sb % G or sh % G or vs.stride(0) != sb // G * D or vs.stride(1) != sh // G * D:
            raise ValueError("grouped v_scale must be laid out [rows/G][D] alongside the codes")
    else:
        if vs.stride(2) != 1 or vs.stride(0) != sb or vs.stride(1) != sh:
            raise ValueError("per-token v_scale must be indexed like the code rows")
    seg.v_scale = vs.data_ptr()
    S = tier.k_packed.shape[2]
    length = getattr(tier, "length", None)
    if length is None and isinstance(tier, (Int4Tier, RotTier)) and tier.max_len is not None and tier.lens is None:
        length = tier.max_len          # padded copy: the valid length is the original S
    seg.len = int(length) if length is not None else S
    seg.max_len = int(tier.max_len) if getattr(tier, "max_len", None) is not None else seg.len
    if tier.lens is not None:
        seg.lens = tier.lens.data_ptr()
    tpr = 128 // min(rbk, rbv)
    seg.n_rows = min(_rows_available(tier.k_packed, rbk), _rows_available(tier.v_packed, rbv)) // tpr * tpr
    keep = [tier.k_packed, tier.v_packed, ks, vs, tier.lens]
    if isinstance(tier, RotTier):
        keep.append(tier.rotation)
    return keep


class DecodePlan:
    """A filled ``fade_decode_desc`` plus its workspace, reusable across calls
    whose tensors keep the same addresses (e.g. inside a CUDA graph)."""

    def __init__(self, q: Tensor, tiers: list, out: Tensor | None = None, sm_scale: float | None = None,
                 n_ctas: int = 0, cu_units: Tensor | None = None, workspace: Tensor | None = None):
        if q.dim() != 4:
            raise ValueError(f"query must be [B, Hq, n_q, D]; got shape {tuple(q.shape)}")
        dev = _lib.require_cuda(q)
        B, Hq, n_q, D = q.shape
        if q.stride(-1) != 1:
            raise ValueError("query must be contiguous in head_dim")
        dtype = q.dtype
        if dtype not in (torch.float16, torch.bfloat16):
            raise ValueError(f"unsupported dtype {dtype}")
        d = _lib.DecodeDesc()
        d.dtype = _lib.dtype_code(dtype)
        d.B, d.Hq, d.D, d.n_q = B, Hq, D, n_q
        d.sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(D)
        d.q = q.data_ptr()
        d.q_sb, d.q_sh, d.q_ss = q.stride(0), q.stride(1), q.stride(2)
        if out is None:
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
        if out.shape != q.shape or out.dtype != dtype or out.stride(-1) != 1:
            raise ValueError("out must match the query's shape and dtype")
        d.out = out.data_ptr()
        d.o_sb, d.o_sh, d.o_ss = out.stride(0), out.stride(1), out.stride(2)
        keep = [q, out]
        Hkv = None
        n = 0
        for t in tiers:
            if t is None:
                continue
            if n >= _lib.MAX_SEGMENTS:
                raise ValueError("too many tiers")
            if isinstance(t, FPTier):
                h = t.k.shape[1]
                keep += _fill_fp(d.seg[n], t, D)
            else:
                h = t.k_scale.shape[1] if getattr(t, "page_table", None) is not None else t.k_packed.shape[1]
                keep += _fill_mid(d.seg[n], t, D, dtype)
                if isinstance(t, RotTier):
                    R = t.rotation
                    if tuple(R.shape) != (D, D):
                        raise ValueError("rotation must be a [D, D] tensor")
                    R = R.to(device=dev, dtype=torch.float32).contiguous()
                    keep.append(R)
                    d.rotation = R.data_ptr()
            if Hkv is None:
                Hkv = h
            elif h != Hkv:
                raise ValueError("all tiers must have the same number of kv heads")
            n += 1
        if Hkv is None:
            raise ValueError("no tiers given")
        if Hq % Hkv:
            raise ValueError(f"Hq={Hq} not divisible by Hkv={Hkv}")
        d.Hkv = Hkv
        d.n_segments = n
        d.n_ctas = int(n_ctas)
        if cu_units is not None:
            d.cu_units = cu_units.data_ptr()
            keep.append(cu_units)
        self.desc = d
        self.out = out
        self._keep = keep
        lib = _lib.load()
        _lib.bind(dev)
        need = lib.fade_decode_attn_workspace_size(ctypes.byref(d))
        if need == 0:
            raise ValueError(
                f"unsupported decode configuration (D={D}, Hq/Hkv*n_q={Hq // Hkv * n_q}, dtype={dtype})"
            )
        if workspace is None or workspace.numel() < need:
            workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        self.workspace = workspace
        self.ws_bytes = workspace.numel()
        self.device = dev

    def rebind(self, q: Tensor, out: Tensor | None = None) -> Tensor:
        """Point the plan at a new query (same shape, dtype and strides) and
        output tensor; the tiers, workspace and sizes stay.  Returns `out`."""
        d = self.desc
        if (tuple(q.shape) != (d.B, d.Hq, d.n_q, d.D) or _lib.dtype_code(q.dtype) != d.dtype
                or (q.stride(0), q.stride(1), q.stride(2)) != (d.q_sb, d.q_sh, d.q_ss)):
            raise ValueError("rebind needs a query with the plan's shape, dtype and strides")
        if out is None:
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
        if out.shape != q.shape or out.dtype != q.dtype or out.stride(-1) != 1:
            raise ValueError("out must match the query's shape and dtype")
        d.q = q.data_ptr()
        d.out = out.data_ptr()
        d.o_sb, d.o_sh, d.o_ss = out.stride(0), out.stride(1), out.stride(2)
        self._keep[0], self._keep[1] = q, out
        self.out = out
        return out

    def run(self) -> Tensor:
        lib = _lib.load()
        st = _lib.bind(self.device)
        _lib.check(lib.fade_decode_attn(ctypes.byref(self.desc), self.workspace.data_ptr(), self.ws_bytes, st),
                   "fade_decode_attn")
        return self.out

    def check_device_errors(self) -> None:
        st = _lib.bind(self.device)
        _lib.check(_lib.load().fade_workspace_check(self.workspace.data_ptr(), self.ws_bytes, st),
                   "fade_decode_attn")


_WS: dict = {}


def _workspace(dev: torch.device) -> Tensor | None:
    key = (dev, torch.cuda.current_stream(dev).cuda_stream)
    return _WS.get(key)


def tiered_decode_attention(q: Tensor, tiers: list, sm_scale: float | None = None, out: Tensor | None = None,
                            n_ctas: int = 0, cu_units: Tensor | None = None) -> Tensor:
    """out[B,Hq,n_q,D] = softmax(q K^T * sm_scale) V over the union of `tiers`.

    GQA: query head ``hq`` reads kv head ``hq // (Hq // Hkv)`` (transformers'
    ``repeat_kv`` convention).  Non-causal over the cached tokens, as a decode
    step is.  Workspace is cached per (device, stream); calls that share a
    stream run in order, so sharing it is safe.
    """
    dev = _lib.require_cuda(q)
    plan = DecodePlan(q, tiers, out=out, sm_scale=sm_scale, n_ctas=n_ctas, cu_units=cu_units,
                      workspace=_workspace(dev))
    _WS[(dev, torch.cuda.current_stream(dev).cuda_stream)] = plan.workspace
    return plan.run()


def fused_int4_sdpa(q: Tensor, k_packed: Tensor, k_scale: Tensor, v_packed: Tensor, v_scale: Tensor,
                    is_causal: bool = False) -> Tensor:
    """Drop-in for the reference's ``fused_int4_sdpa``
    (fade/kernels/fused_int4_attn.py:277-342): attention of q [B, Hq, S_q, D]
    over one bit-packed INT4 segment (k_packed / v_packed [B, Hkv, S_k, D/2],
    k_scale [B, Hkv, 1, D] per channel, v_scale [B, Hkv, S_k, 1] per token),
    sm_scale = 1/sqrt(D), GQA without repeating K/V.  Returns [B, Hq, S_q, D]
    in q's dtype (fp16 for the reference's fp16 inputs).

    ``is_causal`` follows the reference kernel's mask, which is aligned at the
    first key: query m attends keys 0..m (fade/kernels/fused_int4_attn.py:
    166-169).  Each (sequence, query position) then becomes one row of a single
    decode call, all rows of a sequence reading the same code rows (a
    zero-stride batch view) with their own length m + 1.
    Dequantisation rounds each element to the model dtype like the reference's
    dequant_int4 (the reference's Triton kernel keeps it in fp32); both lie
    within the attention tolerance of each other."""
    import math

    dev = _lib.require_cuda(q, k_packed, k_scale, v_packed, v_scale)
    if q.dim() != 4 or k_packed.dim() != 4:
        raise ValueError("q must be [B, H_q, S_q, D] and k_packed [B, H_kv, S_k, D//2]")
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k_packed.shape[1], k_packed.shape[2]
    if Hq % Hkv:
        raise ValueError(f"H_q={Hq} must be a multiple of H_kv={Hkv}")
    sm = 1.0 / math.sqrt(D)
    base = align_tier(Int4Tier(k_packed, k_scale.contiguous(), v_packed, v_scale.contiguous()), D)
    out = torch.empty_like(q)
    if Sk == 0:
        return out.zero_()
    if not is_causal:
        per = max(1, 16 // (Hq // Hkv))          # query positions per call (rows <= 16)
        for s0 in range(0, Sq, per):
            s1 = min(Sq, s0 + per)
            tiered_decode_attention(q[:, :, s0:s1], [base], sm_scale=sm, out=out[:, :, s0:s1])
        return out
    lens = torch.clamp(torch.arange(1, Sq + 1, device=dev, dtype=torch.int32), max=Sk)
    cap = base.k_packed.shape[2]
    for b in range(B):
        def rows(t):                              # the sequence's tensor, once per query position
            return t[b:b + 1].expand(Sq, *t.shape[1:])
        tier = Int4Tier(rows(base.k_packed), rows(base.k_scale), rows(base.v_packed), rows(base.v_scale),
                        lens=lens, max_len=cap)
        qb = q[b].transpose(0, 1).unsqueeze(2)    # [S_q, Hq, 1, D], query position as the batch
        ob = torch.empty((Sq, Hq, 1, D), dtype=q.dtype, device=dev)
        tiered_decode_attention(qb, [tier], sm_scale=sm, out=ob)
        out[b] = ob[:, :, 0].transpose(0, 1)
    return out


_MIDDLE_KERNELS = {"mma_sync": 0, "tcgen05": 1}


def set_middle_kernel(kind: str) -> None:
    """Choose the middle kernel for INT4 K and V at head_dim 128: ``"mma_sync"``
    (default) or ``"tcgen05"`` (tensor-memory accumulators).  Process-wide;
    takes effect for calls made (or graphs captured) afterwards."""
    if kind not in _MIDDLE_KERNELS:
        raise ValueError(f"middle kernel must be one of {sorted(_MIDDLE_KERNELS)}, got {kind!r}")
    _lib.check(_lib.load().fade_set_middle_kernel(_MIDDLE_KERNELS[kind]), "fade_set_middle_kernel")


def get_middle_kernel() -> str:
    code = _lib.load().fade_get_middle_kernel()
    return {v: k for k, v in _MIDDLE_KERNELS.items()}[code]


__all__ = [
    "get_middle_kernel",
    "set_middle_kernel",
    "DecodePlan",
    "FPTier",
    "Int4K2VTier",
    "Int4Tier",
    "RotTier",
    "fused_int4_sdpa",
    "tiered_decode_attention",
]
