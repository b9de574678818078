"""Tiered KV cache for HF transformers on B200 (the reference's ``fade/cache.py``).

``TieredKVCache`` keeps the reference's constructor, tier constants, layer
state, ``update()`` contract (append to the FP16 tier, return K/V of every
retained position in ascending position order), tier reassignment
(``apply_tier_assignment`` / ``apply_tier_assignment_per_sequence``) and
checkpoint format, with every K/V transformation on the sm_100a kernels:

* quantise / pack / dequantise: ``fade_b200.quant`` (bit-exact with
  ``fade/quant.py``), rotated backends: ``fade_b200.rotated_quant``;
* eviction: survivors gathered, un-RoPE'd at their old positions and
  re-RoPE'd at ``0..n_kept-1`` in one kernel pass (``rerope_gather``) instead
  of un-RoPE'ing every token (``fade/cache.py:914-935``);
* decode attention (``decode_attention``): the fused tiered kernel reads the
  sink, recent and quantised middle tiers straight from HBM.  The attention
  function registered by ``fade_b200.patch`` calls it for single-token
  steps, so ``update()`` skips the materialisation there.

Tensors must live on a CUDA device; there is no CPU path.
"""

from __future__ import annotations

import json
import math
import warnings
from dataclasses import dataclass, field
from pathlib import Path

import torch
from torch import Tensor
from transformers.cache_utils import DynamicCache

from fade_b200 import _lib
from fade_b200.attention import FPTier, Int4K2VTier, Int4Tier, RotTier, align_tier, tiered_decode_attention
from fade_b200.backends import QuantBackend, RotatedINT4Backend, SymmetricINT4Backend, get_backend
from fade_b200.quant import (
    DEFAULT_INT2_GROUP_SIZE,
    _pack_int2_last_dim,
    dequant_int4,
    dequant_k_int2,
    dequant_v_int2,
    pad_to_group,
    quant_k_int2,
    quant_k_int4,
    quant_v_int2,
    quant_v_int4,
)
from fade_b200.rope import RopeScheme, Vanilla
from fade_b200.rope_kernels import rerope_gather

DEFAULT_N_SINK: int = 4
DEFAULT_RECENT_WINDOW: int = 128
DEFAULT_INT4_BUDGET: int | None = None
DEFAULT_INT2_BUDGET: int = 0
DEFAULT_ROPE_THETA: float = 10000.0
DEFAULT_FP16_PREALLOC: int = 128
DEFAULT_MAX_DEQUANT_AGE: int | None = None

TIER_FP16: int = 0
TIER_INT4: int = 1
TIER_INT2: int = 2
TIER_EVICT: int = 3
TIER_PQ: int = 4


@dataclass
class LayerState:
    """Per-layer tiers (field names of ``fade/cache.py:52-140``).

    Positions are absolute.  After a reassignment the full cache in position
    order is ``sink | middle (INT4 / backend, then INT2 merged by position) |
    recent``; before one, the FP16 tier holds every token and its first
    ``sink_count`` entries are the sinks.
    """

    sink_k: Tensor | None = None
    sink_v: Tensor | None = None
    sink_pos: Tensor | None = None
    fp16_k: Tensor | None = None
    fp16_v: Tensor | None = None
    fp16_pos: Tensor | None = None
    int4_kq: Tensor | None = None       # packed INT4 K codes [B, H, S, D/2] u8
    int4_ks: Tensor | None = None       # [B, H, 1, D]
    int4_vq: Tensor | None = None       # packed INT4 V [B, H, S, D/2], or int8 INT2 V [B, H, S_pad, D]
    int4_vs: Tensor | None = None       # [B, H, S, 1], or grouped [B, H, S_pad/G, D]
    int4_pos: Tensor | None = None
    int2_kq: Tensor | None = None       # int8 INT2 codes [B, H, S_pad, D]
    int2_ks: Tensor | None = None
    int2_vq: Tensor | None = None
    int2_vs: Tensor | None = None
    int2_pos: Tensor | None = None
    int2_actual_count: int = 0
    int2_group_size: int = DEFAULT_INT2_GROUP_SIZE
    sink_count: int = 0
    next_position: int = 0
    int4_k_deq: Tensor | None = None
    int4_v_deq: Tensor | None = None
    int2_k_deq: Tensor | None = None
    int2_v_deq: Tensor | None = None
    _fp16_buf_k: Tensor | None = None
    _fp16_buf_v: Tensor | None = None
    _fp16_buf_pos: Tensor | None = None
    _fp16_len: int = 0
    _fp16_len_dev: Tensor | None = None   # int32 [B] on the device: _fp16_len, for the decode kernel
    _plan: object = None                  # cached DecodePlan and the tier key it was built for
    _mid_full: tuple | None = None        # (k codes, v codes, v scales) padded to a multiple of 8
                                          # tokens; int4_kq/vq/vs are views of their first rows
    _dequant_age: int = 0
    pq_codes: Tensor | None = None
    pq_v_codes: Tensor | None = None
    pq_pos: Tensor | None = None
    pq_k_deq: Tensor | None = None
    pq_v_deq: Tensor | None = None
    backend_k: dict | None = None
    backend_v: dict | None = None
    backend_pos: Tensor | None = None
    _compressed_bytes: int = 0
    # fused-decode view of the quantised middle (built lazily, dropped on reassignment)
    _kernel_mid: object | None = field(default=None, repr=False)
    _kernel_extra: list | None = field(default=None, repr=False)

    def total_seq_length(self) -> int:
        return sum(int(p.shape[0]) for p in (self.sink_pos, self.fp16_pos, self.int4_pos, self.int2_pos,
                                              self.pq_pos, self.backend_pos) if p is not None)


def _nbytes(t) -> int:
    return int(t.element_size() * t.numel()) if isinstance(t, Tensor) else 0


def _tier_key(t) -> tuple:
    """Identity of a tier's tensors (addresses, shapes, strides): equal keys
    mean a DecodePlan built for one describes the other."""
    out = [type(t).__name__]
    for name in ("k", "v", "k_packed", "k_scale", "v_packed", "v_scale", "lens", "rotation"):
        x = getattr(t, name, None)
        if isinstance(x, torch.Tensor):
            out.append((name, x.data_ptr(), tuple(x.shape), tuple(x.stride())))
    for name in ("group", "length", "max_len", "bits"):
        if hasattr(t, name):
            out.append((name, getattr(t, name)))
    return tuple(out)


class TieredKVCache(DynamicCache):
    """Tiered KV cache: FP16 sinks + recent window, INT4 (or backend) middle,
    optional INT2 tier, eviction with re-RoPE.

    Invariants (as the reference's): a position lives in at most one tier;
    absolute positions are never renumbered except by eviction, which re-RoPEs
    survivors to contiguous positions; ``update()`` returns every retained
    position in ascending order.  ``apply_tier_assignment`` shares one tier
    vector across the batch (lockstep decoding); the per-sequence variant
    assigns each row independently and pads rows to the longest.
    """

    def __init__(
        self,
        n_sink: int = DEFAULT_N_SINK,
        recent_window: int = DEFAULT_RECENT_WINDOW,
        int4_budget: int | None = DEFAULT_INT4_BUDGET,
        int2_budget: int = DEFAULT_INT2_BUDGET,
        dtype: torch.dtype = torch.float16,
        cache_dequant: bool = True,
        rope_theta: float = DEFAULT_ROPE_THETA,
        head_dim: int | None = None,
        batch_size: int | None = None,
        rope_scheme: RopeScheme | None = None,
        middle_k_bits: int = 4,
        middle_v_bits: int = 4,
        quant_backend: str | QuantBackend = "int4",
        *,
        v_int2_group_size: int = DEFAULT_INT2_GROUP_SIZE,
    ) -> None:
        super().__init__()
        # tokens per scale group of the 2-bit V middle (middle_v_bits=2); the
        # reference fixes it at DEFAULT_INT2_GROUP_SIZE (fade/cache.py:986)
        self.v_int2_group_size = int(v_int2_group_size)
        self.n_sink = n_sink
        self.recent_window = recent_window
        self.int4_budget = int4_budget
        self.int2_budget = int2_budget
        self.dtype = dtype
        self.cache_dequant = cache_dequant
        self.rope_theta = rope_theta
        self.head_dim = head_dim
        self.batch_size = batch_size
        self.max_dequant_age = DEFAULT_MAX_DEQUANT_AGE
        self.middle_k_bits = middle_k_bits
        self.middle_v_bits = middle_v_bits
        self._quant_backend: QuantBackend = (
            get_backend(quant_backend, head_dim=head_dim or 64) if isinstance(quant_backend, str) else quant_backend
        )
        self._rope_scheme = rope_scheme
        self._skip_layers: set[int] = set()
        self._layers: list[LayerState] = []
        # set by fade_b200.patch when the model's attention reads the tiers itself
        self.fused_decode = False

    # ------------------------------------------------------------------ misc
    def set_skip_layers(self, layer_indices) -> None:
        """Layers kept as plain FP16 passthrough (e.g. linear-attention layers)."""
        self._skip_layers = set(layer_indices)

    @property
    def managed_layers(self) -> set[int]:
        return {i for i in range(len(self._layers)) if i not in self._skip_layers}

    def is_managed(self, layer_idx: int) -> bool:
        return layer_idx not in self._skip_layers

    def enable_compile(self, **compile_kwargs) -> None:
        """Accepted for API compatibility; the materialisation and the decode
        attention already run as fused CUDA kernels, so nothing is compiled."""
        warnings.warn("enable_compile() is a no-op: the hot path is hand-written CUDA", RuntimeWarning,
                      stacklevel=2)

    def set_codebooks(self, k_codebook, v_codebook=None) -> None:
        """Product-quantisation codebooks (the reference's TIER_PQ) are not
        part of this build."""
        raise NotImplementedError("TIER_PQ (product-quantisation codebooks) is not supported by fade_b200")

    def _ensure_rope_scheme(self) -> RopeScheme:
        if self._rope_scheme is None:
            self._rope_scheme = Vanilla(theta=self.rope_theta, head_dim=self.head_dim or 64)
        return self._rope_scheme

    @property
    def rope_scheme(self) -> RopeScheme:
        return self._ensure_rope_scheme()

    def _compute_cos_sin(self, positions: Tensor, device) -> tuple[Tensor, Tensor]:
        return self._ensure_rope_scheme().compute_cos_sin(positions, device, model_dtype=self.dtype)

    @staticmethod
    def _streamingllm_positions(total: int, device) -> Tensor:
        return torch.arange(total, device=device, dtype=torch.long)

    # ------------------------------------------------------- HF cache API
    def update(self, key_states: Tensor, value_states: Tensor, layer_idx: int,
               cache_kwargs: dict | None = None) -> tuple[Tensor, Tensor]:
        """Append new K/V (post-RoPE) to the FP16 tier and return the full
        cache.  Under the fused attention function a single-token step returns
        the new token only (the attention reads the tiers)."""
        if key_states.dim() != 4:
            raise ValueError(f"key_states must be [B, H, S, D]; got shape {tuple(key_states.shape)}")
        if key_states.shape != value_states.shape:
            raise ValueError(
                f"K/V shape mismatch: {tuple(key_states.shape)} vs {tuple(value_states.shape)}")
        _lib.require_cuda(key_states, value_states)
        B = int(key_states.shape[0])
        if self.batch_size is None:
            self.batch_size = B
        elif self.batch_size != B:
            raise ValueError(f"batch size mismatch: cache pinned to B={self.batch_size} but got B={B}")
        if self.head_dim is None:
            self.head_dim = int(key_states.shape[-1])
        self._ensure_layer(layer_idx)
        self._append_fp16(key_states, value_states, layer_idx)
        if self.fused_decode and key_states.shape[-2] == 1 and self.is_managed(layer_idx):
            return key_states, value_states
        return self._materialize(layer_idx)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._layers[layer_idx].total_seq_length() if layer_idx < len(self._layers) else 0

    def get_mask_sizes(self, cache_position, layer_idx: int = 0) -> tuple[int, int]:
        """(kv_length, kv_offset) for the attention mask."""
        q = cache_position if isinstance(cache_position, int) else int(cache_position.shape[0])
        return self.get_seq_length(layer_idx) + q, 0

    def __len__(self) -> int:
        return len(self._layers)

    # ------------------------------------------------------------ bytes
    def storage_bytes(self) -> int:
        """Bytes held for K/V in all tiers, dequantised caches included."""
        names = ("fp16_k", "fp16_v", "int4_kq", "int4_vq", "int4_ks", "int4_vs", "int4_k_deq", "int4_v_deq",
                 "int2_kq", "int2_vq", "int2_ks", "int2_vs", "int2_k_deq", "int2_v_deq")
        return sum(_nbytes(getattr(s, n)) for s in self._layers for n in names)

    @staticmethod
    def _layer_compressed_bytes(state: LayerState) -> int:
        names = ("sink_k", "sink_v", "fp16_k", "fp16_v", "int4_kq", "int4_vq", "int4_ks", "int4_vs",
                 "int2_kq", "int2_vq", "int2_ks", "int2_vs")
        total = sum(_nbytes(getattr(state, n)) for n in names)
        for d in (state.backend_k, state.backend_v):
            if isinstance(d, dict):
                total += sum(_nbytes(v) for v in d.values())
        return total

    def compressed_storage_bytes(self) -> int:
        """Bytes of the at-rest compressed form (no dequantised caches)."""
        if self._layers and any(s._compressed_bytes > 0 for s in self._layers):
            return sum(s._compressed_bytes for s in self._layers)
        return sum(self._layer_compressed_bytes(s) for s in self._layers)

    # ------------------------------------------------------- checkpoint
    _LAYER_TENSOR_KEYS = ("sink_k", "sink_v", "sink_pos", "fp16_k", "fp16_v", "fp16_pos", "int4_kq", "int4_ks",
                          "int4_vq", "int4_vs", "int4_pos", "int2_kq", "int2_ks", "int2_vq", "int2_vs", "int2_pos")
    _LAYER_SCALAR_KEYS = ("int2_actual_count", "int2_group_size", "sink_count", "next_position")

    def cache_state_dict(self) -> dict:
        """The compressed form as a plain dict for ``torch.save`` (the
        reference's keys: ``layer.{i}.{field}``)."""
        sd: dict = {"n_layers": len(self._layers), "n_sink": self.n_sink, "recent_window": self.recent_window,
                    "int4_budget": self.int4_budget, "int2_budget": self.int2_budget,
                    "batch_size": self.batch_size, "head_dim": self.head_dim, "dtype": str(self.dtype)}
        for i, st in enumerate(self._layers):
            for key in self._LAYER_TENSOR_KEYS:
                val = getattr(st, key)
                if val is not None:
                    sd[f"layer.{i}.{key}"] = val.cpu()
            for key in self._LAYER_SCALAR_KEYS:
                sd[f"layer.{i}.{key}"] = getattr(st, key)
        return sd

    def load_cache_state_dict(self, sd: dict, device: torch.device | str | None = None) -> None:
        """Restore layer state saved by ``cache_state_dict``; tensors go to
        ``device`` (default: the current CUDA device)."""
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._layers = []
        for i in range(sd["n_layers"]):
            st = LayerState()
            for key in self._LAYER_TENSOR_KEYS:
                val = sd.get(f"layer.{i}.{key}")
                if val is not None:
                    setattr(st, key, val.to(dev))
            for key in self._LAYER_SCALAR_KEYS:
                val = sd.get(f"layer.{i}.{key}")
                if val is not None:
                    setattr(st, key, val)
            self._layers.append(st)
        if sd.get("batch_size") is not None:
            self.batch_size = sd["batch_size"]
        if sd.get("head_dim") is not None:
            self.head_dim = sd["head_dim"]

    def dump_debug(self, path) -> None:
        """JSON snapshot of tier membership and positions per layer."""
        def n(p):
            return int(p.shape[0]) if p is not None else 0

        layers = []
        for i, st in enumerate(self._layers):
            d = {"layer_idx": i, "sink_count": st.sink_count, "next_position": st.next_position,
                 "fp16_count": n(st.fp16_pos), "int4_count": n(st.int4_pos), "int2_count": n(st.int2_pos),
                 "int2_actual_count": st.int2_actual_count, "total_seq_length": st.total_seq_length()}
            for key, p in (("sink_positions", st.sink_pos), ("fp16_positions", st.fp16_pos),
                           ("int4_positions", st.int4_pos), ("int2_positions", st.int2_pos)):
                if p is not None:
                    d[key] = p.tolist()
            layers.append(d)
        snap = {"n_layers": len(self._layers), "n_sink": self.n_sink, "recent_window": self.recent_window,
                "int4_budget": self.int4_budget, "int2_budget": self.int2_budget, "batch_size": self.batch_size,
                "head_dim": self.head_dim, "layers": layers}
        Path(path).write_text(json.dumps(snap, indent=2), encoding="utf-8")

    # --------------------------------------------------------- internals
    def _ensure_layer(self, layer_idx: int) -> None:
        while len(self._layers) <= layer_idx:
            self._layers.append(LayerState())

    def _append_fp16(self, k: Tensor, v: Tensor, layer_idx: int) -> None:
        """Append to a pre-allocated FP16 buffer that doubles when full;
        ``fp16_k/v/pos`` are views of its filled prefix."""
        st = self._layers[layer_idx]
        n = int(k.shape[-2])
        pos = torch.arange(st.next_position, st.next_position + n, device=k.device)
        st.next_position += n
        B, H, _, D = k.shape
        if st._fp16_buf_k is None:
            have = int(st.fp16_k.shape[-2]) if st.fp16_k is not None else 0
            cap = max(DEFAULT_FP16_PREALLOC, have + n)
            bk = torch.empty(B, H, cap, D, dtype=k.dtype, device=k.device)
            bv = torch.empty(B, H, cap, D, dtype=v.dtype, device=v.device)
            bp = torch.empty(cap, dtype=torch.long, device=k.device)
            if have:
                bk[:, :, :have] = st.fp16_k
                bv[:, :, :have] = st.fp16_v
                bp[:have] = st.fp16_pos
            st._fp16_buf_k, st._fp16_buf_v, st._fp16_buf_pos, st._fp16_len = bk, bv, bp, have
        cur, cap = st._fp16_len, st._fp16_buf_k.shape[-2]
        if cur + n > cap:
            new_cap = max(2 * cap, cur + n)
            for name in ("_fp16_buf_k", "_fp16_buf_v"):
                old = getattr(st, name)
                nb = torch.empty(B, H, new_cap, D, dtype=old.dtype, device=old.device)
                nb[:, :, :cur] = old[:, :, :cur]
                setattr(st, name, nb)
            nbp = torch.empty(new_cap, dtype=torch.long, device=k.device)
            nbp[:cur] = st._fp16_buf_pos[:cur]
            st._fp16_buf_pos = nbp
        st._fp16_buf_k[:, :, cur:cur + n] = k
        st._fp16_buf_v[:, :, cur:cur + n] = v
        st._fp16_buf_pos[cur:cur + n] = pos
        st._fp16_len = cur + n
        self._sync_fp16_len(st)
        st.fp16_k = st._fp16_buf_k[:, :, :st._fp16_len]
        st.fp16_v = st._fp16_buf_v[:, :, :st._fp16_len]
        st.fp16_pos = st._fp16_buf_pos[:st._fp16_len]
        st._dequant_age += 1

    def _materialize(self, layer_idx: int) -> tuple[Tensor, Tensor]:
        parts_k, parts_v = self._assemble_parts(self._layers[layer_idx], want_positions=False)
        if not parts_k:
            raise RuntimeError(f"No cache state for layer {layer_idx}")
        return torch.cat(parts_k, dim=-2), torch.cat(parts_v, dim=-2)

    def _all_in_position_order(self, layer_idx: int) -> tuple[Tensor, Tensor, Tensor]:
        pk, pv, pp = self._assemble_parts(self._layers[layer_idx], want_positions=True)
        if not pk:
            raise RuntimeError(f"No cache state for layer {layer_idx}")
        return torch.cat(pk, dim=-2), torch.cat(pv, dim=-2), torch.cat(pp, dim=0)

    def _assemble_parts(self, st: LayerState, want_positions: bool):
        """Tier segments in the order sink | middle | recent (the reference's
        ``_assemble_parts``, ``fade/cache.py:714-790``)."""
        pk, pv, pp = [], [], []
        nsk = st.sink_count
        if st.sink_k is not None:
            pk.append(st.sink_k)
            pv.append(st.sink_v)
            pp.append(st.sink_pos)
        elif st.fp16_k is not None and nsk > 0:
            pk.append(st.fp16_k[..., :nsk, :])
            pv.append(st.fp16_v[..., :nsk, :])
            pp.append(st.fp16_pos[:nsk])
        mk, mv, mp = [], [], []
        if st.int4_kq is not None:
            k4, v4 = self._get_int4_dequant(st)
            mk.append(k4)
            mv.append(v4)
            mp.append(st.int4_pos)
        if st.backend_k is not None:
            mk.append(self._quant_backend.decompress_k(st.backend_k, dtype=self.dtype))
            mv.append(self._quant_backend.decompress_v(st.backend_v, dtype=self.dtype))
            mp.append(st.backend_pos)
        if st.int2_kq is not None:
            k2, v2 = self._get_int2_dequant(st)
            mk.append(k2)
            mv.append(v2)
            mp.append(st.int2_pos)
        if len(mk) == 1:
            pk.append(mk[0])
            pv.append(mv[0])
            pp.append(mp[0])
        elif mk:
            order = torch.cat(mp).argsort()
            pk.append(torch.cat(mk, dim=-2).index_select(-2, order))
            pv.append(torch.cat(mv, dim=-2).index_select(-2, order))
            pp.append(torch.cat(mp)[order])
        if st.fp16_k is not None:
            start = 0 if st.sink_k is not None else nsk
            if start < int(st.fp16_k.shape[-2]):
                pk.append(st.fp16_k[..., start:, :])
                pv.append(st.fp16_v[..., start:, :])
                pp.append(st.fp16_pos[start:])
        return (pk, pv, pp) if want_positions else (pk, pv)

    def _get_int4_dequant(self, st: LayerState) -> tuple[Tensor, Tensor]:
        if (self.max_dequant_age is not None and st._dequant_age > self.max_dequant_age
                and st.int4_k_deq is not None):
            st.int4_k_deq = st.int4_v_deq = None
        if self.cache_dequant and st.int4_k_deq is not None:
            return st.int4_k_deq, st.int4_v_deq
        k = dequant_int4(st.int4_kq, st.int4_ks, dtype=self.dtype)
        if self.middle_v_bits == 4:
            v = dequant_int4(st.int4_vq, st.int4_vs, dtype=self.dtype)
        else:
            v = dequant_v_int2(st.int4_vq, st.int4_vs, group_size=self.v_int2_group_size, dtype=self.dtype)
            n = int(st.int4_pos.shape[0]) if st.int4_pos is not None else 0
            if 0 < n < v.shape[-2]:
                v = v[..., :n, :]
        if self.cache_dequant:
            st.int4_k_deq, st.int4_v_deq, st._dequant_age = k, v, 0
        return k, v

    def _get_int2_dequant(self, st: LayerState) -> tuple[Tensor, Tensor]:
        if self.cache_dequant and st.int2_k_deq is not None:
            return st.int2_k_deq, st.int2_v_deq
        gs = st.int2_group_size
        k = dequant_k_int2(st.int2_kq, st.int2_ks, group_size=gs, dtype=self.dtype)
        v = dequant_v_int2(st.int2_vq, st.int2_vs, group_size=gs, dtype=self.dtype)
        n = st.int2_actual_count
        if 0 < n < k.shape[-2]:
            k, v = k[..., :n, :], v[..., :n, :]
        if self.cache_dequant:
            st.int2_k_deq, st.int2_v_deq = k, v
        return k, v

    # ---------------------------------------------------- fused decode
    def _kernel_middle(self, st: LayerState):
        """The middle tier as the fused kernel reads it (built once per
        reassignment): INT4, INT4 K + packed grouped INT2 V, or rotated
        2/4-bit codes, padded so each row's segment starts on a 128-byte code
        row.  Tokens the kernel has no format for (the INT2 tier, 3-bit
        rotated codes) are dequantised once into an extra FP tier."""
        if st._kernel_mid is not None or st._kernel_extra is not None:
            return st._kernel_mid, st._kernel_extra or []
        D = int(self.head_dim)
        mid, extra = None, []
        if st.int4_kq is not None:
            n = int(st.int4_kq.shape[-2])
            full = st._mid_full
            if full is None or full[0].data_ptr() != st.int4_kq.data_ptr():
                full = None                # tiers replaced since (e.g. a loaded checkpoint)
            if self.middle_v_bits == 4:
                if full is not None:       # the padded buffers the tiers are views of: no copy
                    mid = Int4Tier(full[0], st.int4_ks, full[1], full[2], max_len=n)
                else:
                    mid = Int4Tier(st.int4_kq, st.int4_ks, st.int4_vq, st.int4_vs)
            else:
                kq = full[0] if full is not None else st.int4_kq
                mid = Int4K2VTier(kq, st.int4_ks, _pack_int2_last_dim(st.int4_vq), st.int4_vs,
                                  group=self.v_int2_group_size, length=n)
        elif st.backend_k is not None:
            be = self._quant_backend
            if isinstance(be, RotatedINT4Backend) and be.bits in (2, 4):
                R = be.rotation(st.backend_k["packed"].device)
                mid = RotTier(st.backend_k["packed"], st.backend_k["scale"], st.backend_v["packed"],
                              st.backend_v["scale"], bits=be.bits, rotation=R)
            else:
                extra.append(FPTier(be.decompress_k(st.backend_k, dtype=self.dtype),
                                    be.decompress_v(st.backend_v, dtype=self.dtype)))
        if mid is not None:
            mid = align_tier(mid, D)
        if st.int2_kq is not None:
            k2, v2 = self._get_int2_dequant(st)
            extra.append(FPTier(k2.contiguous(), v2.contiguous()))
        st._kernel_mid, st._kernel_extra = mid, extra
        return mid, extra

    def decode_tiers(self, layer_idx: int) -> list:
        """The layer's tiers for ``tiered_decode_attention`` (order-free)."""
        st = self._layers[layer_idx]
        tiers = []
        if st.sink_k is not None:
            tiers.append(FPTier(st.sink_k, st.sink_v))
        mid, extra = self._kernel_middle(st)
        if mid is not None:
            tiers.append(mid)
        tiers.extend(extra)
        if st._fp16_buf_k is not None and st._fp16_len > 0:
            # the whole buffer with its device fill level: stable across steps
            tiers.append(FPTier(st._fp16_buf_k, st._fp16_buf_v, lens=st._fp16_len_dev))
        elif st.fp16_k is not None and st.fp16_k.shape[-2] > 0:
            tiers.append(FPTier(st.fp16_k, st.fp16_v))   # before a reassignment: sinks included
        return tiers

    def decode_attention(self, layer_idx: int, query: Tensor, scaling: float | None = None,
                         out: Tensor | None = None) -> Tensor:
        """softmax(q K^T * scaling) V over every retained token of the layer,
        from the compressed tiers: query [B, Hq, n_q, D] -> [B, Hq, n_q, D].

        The layer keeps one DecodePlan (descriptor + workspace) between
        reassignments; a call whose tiers are unchanged only re-points it at
        the new query and output."""
        from fade_b200 import attention as att

        st = self._layers[layer_idx]
        tiers = self.decode_tiers(layer_idx)
        key = (tuple(query.shape), tuple(query.stride()), query.dtype, scaling, tuple(_tier_key(t) for t in tiers))
        if st._plan is not None and st._plan[0] == key:
            plan = st._plan[1]
            plan.rebind(query, out)
            return plan.run()
        dev = query.device
        plan = att.DecodePlan(query, tiers, out=out, sm_scale=scaling, workspace=att._workspace(dev))
        att._WS[(dev, torch.cuda.current_stream(dev).cuda_stream)] = plan.workspace
        st._plan = (key, plan)
        return plan.run()

    # -------------------------------------------------- tier management
    def _rerope(self, k: Tensor, v: Tensor, pos: Tensor, keep_idx: Tensor):
        """Survivors at ``keep_idx``: un-RoPE at ``pos``, re-RoPE at 0..n-1."""
        n = int(keep_idx.numel())
        new_pos = self._streamingllm_positions(n, pos.device)
        scheme = self._ensure_rope_scheme()
        cos_all, sin_all = self._compute_cos_sin(torch.cat([pos, new_pos]), pos.device)
        S = int(pos.shape[0])
        D = k.shape[-1]
        co, so = cos_all.reshape(-1, D)[:S], sin_all.reshape(-1, D)[:S]
        cn, sn = cos_all.reshape(-1, D)[S:], sin_all.reshape(-1, D)[S:]
        k2, v2 = rerope_gather(k.contiguous(), v.contiguous(), keep_idx, co, so, cn, sn,
                               apply_rope=scheme.is_rope)
        return k2, v2, new_pos

    def _quant_int4_tier(self, st: LayerState, k_sub: Tensor, v_sub: Tensor, pos: Tensor) -> None:
        if isinstance(self._quant_backend, SymmetricINT4Backend):
            # Quantise over the tokens padded with zeros to a multiple of 8 (of
            # the V group with 2-bit V): every (b, h) segment then starts on a
            # 128-byte code row and the decode kernel streams these buffers as
            # they are.  Zero tokens change no per-channel K absmax and get
            # their own V scales; the stored tiers are views of the first n.
            n = int(k_sub.shape[-2])
            mult = 8 if self.middle_v_bits == 4 else self.v_int2_group_size
            n_pad = -(-n // mult) * mult
            if n_pad != n:
                z = k_sub.new_zeros(k_sub.shape[:2] + (n_pad - n, k_sub.shape[-1]))
                k_pad, v_pad = torch.cat([k_sub, z], dim=-2), torch.cat([v_sub, z], dim=-2)
            else:
                k_pad, v_pad = k_sub, v_sub
            kq, st.int4_ks = quant_k_int4(k_pad)
            st.int4_kq = kq[:, :, :n]
            if self.middle_v_bits == 4:
                vq, vs = quant_v_int4(v_pad)
                st.int4_vq, st.int4_vs = vq[:, :, :n], vs[:, :, :n]
                st._mid_full = (kq, vq, vs)
            else:
                st.int4_vq, st.int4_vs = quant_v_int2(v_pad, group_size=self.v_int2_group_size)
                st._mid_full = (kq, None, None)
            st.int4_pos = pos
            st.backend_k = st.backend_v = st.backend_pos = None
        else:
            st.backend_k = self._quant_backend.compress_k(k_sub)
            st.backend_v = self._quant_backend.compress_v(v_sub)
            st.backend_pos = pos
            st.int4_kq = st.int4_vq = st.int4_ks = st.int4_vs = st.int4_pos = None

    def _reseed_fp16_buffer(self, st: LayerState) -> None:
        n = int(st.fp16_k.shape[-2]) if st.fp16_k is not None else 0
        if n > 0 and st._fp16_buf_k is not None and n <= st._fp16_buf_k.shape[-2]:
            # fp16_k/v/pos are fresh tensors here (gathered), never views of the buffer
            st._fp16_buf_k[:, :, :n] = st.fp16_k
            st._fp16_buf_v[:, :, :n] = st.fp16_v
            st._fp16_buf_pos[:n] = st.fp16_pos
            st._fp16_len = n
            self._sync_fp16_len(st)
            st.fp16_k, st.fp16_v = st._fp16_buf_k[:, :, :n], st._fp16_buf_v[:, :, :n]
            st.fp16_pos = st._fp16_buf_pos[:n]
        else:
            st._fp16_buf_k = st._fp16_buf_v = st._fp16_buf_pos = None
            st._fp16_len = 0

    def _invalidate(self, st: LayerState) -> None:
        st.int4_k_deq = st.int4_v_deq = st.int2_k_deq = st.int2_v_deq = None
        st.pq_k_deq = st.pq_v_deq = None
        st._kernel_mid = st._kernel_extra = None
        st._plan = None

    @staticmethod
    def _sync_fp16_len(st: LayerState) -> None:
        """The recent tier's fill level as a device int32 [B] (the decode
        kernel reads the fixed-capacity buffer up to it, so one plan serves
        every step between reassignments)."""
        B = int(st._fp16_buf_k.shape[0])
        if st._fp16_len_dev is None or st._fp16_len_dev.numel() != B or \
                st._fp16_len_dev.device != st._fp16_buf_k.device:
            st._fp16_len_dev = torch.empty(B, dtype=torch.int32, device=st._fp16_buf_k.device)
        st._fp16_len_dev.fill_(st._fp16_len)

    def apply_tier_assignment(self, layer_idx: int, tiers: Tensor, scores: Tensor | None = None, *,
                              counts: tuple[int, int, int] | None = None) -> None:
        """Move tokens between tiers (``fade/cache.py:881-1057``): ``tiers``
        [S] in ascending position order with values TIER_FP16 / INT4 / INT2 /
        EVICT.  Evicting re-RoPEs the survivors to contiguous positions and
        resets ``next_position``; FP16 survivors split into the first
        ``n_sink`` sinks and the recent tier.

        ``counts`` (an extension; the reference has no such argument): the
        number of FP16, INT4 and INT2 entries of ``tiers`` when the caller
        knows them, as after ``_assign_one_layer`` (``assign_counts`` gives
        them from the budgets).  The tiers' positions are then grouped with
        one device sort instead of boolean masks and ``nonzero``, and the call
        makes no host synchronisation (the reference synchronises on every
        reassignment, ``fade/cache.py:912``).  Wrong counts give wrong tiers;
        TIER_PQ entries are not detected on this path."""
        del scores
        st = self._layers[layer_idx]
        k_full, v_full, pos_full = self._all_in_position_order(layer_idx)
        S = int(pos_full.shape[0])
        if int(tiers.shape[0]) != S:
            raise ValueError(f"tiers length {int(tiers.shape[0])} != cache length {S} for layer {layer_idx}")
        tiers = tiers.to(pos_full.device)
        if counts is None:
            if bool((tiers == TIER_PQ).any()):
                raise NotImplementedError("TIER_PQ (product-quantisation codebooks) is not supported by fade_b200")
            keep = tiers != TIER_EVICT
            n_kept = int(keep.sum().item())
            if n_kept < S:
                keep_idx = keep.nonzero(as_tuple=False).squeeze(-1)
                k_full, v_full, pos_full = self._rerope(k_full, v_full, pos_full, keep_idx)
                tiers = tiers[keep]
                st.next_position = n_kept
            groups = None
        else:
            n_fp, n_i4, n_i2 = (int(c) for c in counts)
            if min(n_fp, n_i4, n_i2) < 0 or n_fp + n_i4 + n_i2 > S:
                raise ValueError(f"counts {counts} do not fit a cache of length {S}")
            n_kept = n_fp + n_i4 + n_i2
            if n_kept < S:
                # kept positions in ascending order: evicted ones sort last
                ar = torch.arange(S, device=tiers.device)
                keep_idx = torch.argsort((tiers == TIER_EVICT).to(torch.int64) * S + ar)[:n_kept]
                keep_idx = keep_idx.sort().values
                k_full, v_full, pos_full = self._rerope(k_full, v_full, pos_full, keep_idx)
                tiers = tiers.index_select(0, keep_idx)
                st.next_position = n_kept
            # every tier's positions, ascending, as consecutive runs of one sort
            rank = torch.full_like(tiers, 3)
            rank = torch.where(tiers == TIER_FP16, torch.zeros_like(rank), rank)
            rank = torch.where(tiers == TIER_INT4, torch.ones_like(rank), rank)
            rank = torch.where(tiers == TIER_INT2, torch.full_like(rank, 2), rank)
            order = torch.argsort(rank * n_kept + torch.arange(n_kept, device=tiers.device))
            groups = (order[:n_fp], order[n_fp:n_fp + n_i4], order[n_fp + n_i4:n_kept])

        def sel(t, idx, dim):
            return t.index_select(dim, idx).contiguous()

        def tier_idx(which: int, tier: int) -> Tensor:
            if groups is not None:
                return groups[which]
            return (tiers == tier).nonzero(as_tuple=False).squeeze(-1)

        fp_idx = tier_idx(0, TIER_FP16)
        if fp_idx.numel() > 0:
            fk, fv, fpos = sel(k_full, fp_idx, -2), sel(v_full, fp_idx, -2), sel(pos_full, fp_idx, 0)
            ns = min(self.n_sink, int(fp_idx.numel()))
            if ns > 0:
                st.sink_k, st.sink_v, st.sink_pos = fk[..., :ns, :], fv[..., :ns, :], fpos[:ns]
            else:
                st.sink_k = st.sink_v = st.sink_pos = None
            if ns < int(fp_idx.numel()):
                st.fp16_k, st.fp16_v, st.fp16_pos = fk[..., ns:, :], fv[..., ns:, :], fpos[ns:]
            else:
                st.fp16_k = st.fp16_v = st.fp16_pos = None
        else:
            st.fp16_k = st.fp16_v = st.fp16_pos = None
            st.sink_k = st.sink_v = st.sink_pos = None
        self._reseed_fp16_buffer(st)

        i4 = tier_idx(1, TIER_INT4)
        if i4.numel() > 0:
            self._quant_int4_tier(st, sel(k_full, i4, -2), sel(v_full, i4, -2), sel(pos_full, i4, 0))
        else:
            st.int4_kq = st.int4_vq = st.int4_ks = st.int4_vs = st.int4_pos = None
            st.backend_k = st.backend_v = st.backend_pos = None

        i2 = tier_idx(2, TIER_INT2)
        if i2.numel() > 0:
            gs = DEFAULT_INT2_GROUP_SIZE
            k2, _ = pad_to_group(sel(k_full, i2, -2), gs)
            v2, _ = pad_to_group(sel(v_full, i2, -2), gs)
            st.int2_kq, st.int2_ks = quant_k_int2(k2, group_size=gs)
            st.int2_vq, st.int2_vs = quant_v_int2(v2, group_size=gs)
            st.int2_pos = sel(pos_full, i2, 0)
            st.int2_actual_count = int(i2.numel())
            st.int2_group_size = gs
        else:
            st.int2_kq = st.int2_vq = st.int2_ks = st.int2_vs = st.int2_pos = None
            st.int2_actual_count = 0
        st.pq_codes = st.pq_v_codes = st.pq_pos = None
        self._invalidate(st)
        st._compressed_bytes = self._layer_compressed_bytes(st)
        st.sink_count = int(st.sink_pos.shape[0]) if st.sink_pos is not None else 0

    def apply_tier_assignment_per_sequence(self, layer_idx: int, tiers_per_row: Tensor,
                                           scores: Tensor | None = None) -> None:
        """Per-row tier assignment (``fade/cache.py:1059-1230``): each row is
        evicted / split independently, then FP16 and INT4 tiers are padded
        with zero tokens to the longest row (positions of row 0).  INT2 is not
        kept on this path (as in the reference)."""
        del scores
        st = self._layers[layer_idx]
        k_full, v_full, pos_full = self._all_in_position_order(layer_idx)
        B, H, _, D = k_full.shape
        S = int(pos_full.shape[0])
        if tiers_per_row.dim() != 2 or tiers_per_row.shape[0] != B:
            raise ValueError(f"tiers_per_row must be [B={B}, S={S}], got {tuple(tiers_per_row.shape)}")
        if tiers_per_row.shape[1] != S:
            raise ValueError(f"tiers_per_row S dim {tiers_per_row.shape[1]} != cache length {S}")
        dev = k_full.device
        tiers_per_row = tiers_per_row.to(dev)
        fp_rows, i4_rows = [], []
        min_next = S
        for b in range(B):
            t = tiers_per_row[b]
            rk, rv, rpos = k_full[b:b + 1], v_full[b:b + 1], pos_full
            keep = t != TIER_EVICT
            n_kept = int(keep.sum().item())
            if n_kept < S:
                rk, rv, rpos = self._rerope(rk, rv, pos_full, keep.nonzero(as_tuple=False).squeeze(-1))
                t = t[keep]
                min_next = min(min_next, n_kept)
            for tier_id, rows in ((TIER_FP16, fp_rows), (TIER_INT4, i4_rows)):
                idx = (t == tier_id).nonzero(as_tuple=False).squeeze(-1)
                rows.append((rk.index_select(-2, idx), rv.index_select(-2, idx), rpos[idx]))

        def stack(rows):
            L = max(r[0].shape[-2] for r in rows)
            if L == 0:
                return None
            ks, vs = [], []
            for rk, rv, _ in rows:
                gap = L - rk.shape[-2]
                if gap:
                    z = torch.zeros(1, H, gap, D, dtype=rk.dtype, device=dev)
                    rk, rv = torch.cat([rk, z], dim=-2), torch.cat([rv, z], dim=-2)
                ks.append(rk)
                vs.append(rv)
            return torch.cat(ks, dim=0), torch.cat(vs, dim=0), rows[0][2][:L]

        fp = stack(fp_rows)
        st.sink_k = st.sink_v = st.sink_pos = None
        if fp is not None:
            st.fp16_k, st.fp16_v, st.fp16_pos = fp
        else:
            st.fp16_k = st.fp16_v = st.fp16_pos = None
        self._reseed_fp16_buffer(st)
        i4 = stack(i4_rows)
        if i4 is not None:
            self._quant_int4_tier(st, i4[0].contiguous(), i4[1].contiguous(), i4[2])
        else:
            st.int4_kq = st.int4_vq = st.int4_ks = st.int4_vs = st.int4_pos = None
            st.backend_k = st.backend_v = st.backend_pos = None
        st.int2_kq = st.int2_vq = st.int2_ks = st.int2_vs = st.int2_pos = None
        st.int2_actual_count = 0
        st.pq_codes = st.pq_v_codes = st.pq_pos = None
        self._invalidate(st)
        st.next_position = min_next
        st.sink_count = min(self.n_sink, int(st.fp16_pos.shape[0])) if st.fp16_pos is not None else 0
        st._compressed_bytes = self._layer_compressed_bytes(st)


__all__ = [
    "DEFAULT_N_SINK",
    "DEFAULT_RECENT_WINDOW",
    "LayerState",
    "TIER_EVICT",
    "TIER_FP16",
    "TIER_INT2",
    "TIER_INT4",
    "TIER_PQ",
    "TieredKVCache",
]
