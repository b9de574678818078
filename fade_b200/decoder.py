"""Multi-layer tiered decode step on device, with CUDA-graph capture.

``TieredDecoder`` keeps, per layer, the FADE "safe" tier layout for a batch in
lockstep (the reference's shared-tier batching, fade/cache.py:136-161):

* FP16/BF16 attention sinks          sink_k/v   [B, Hkv, n_sink, D]
* FP16/BF16 recent window (a ring)   ring_k/v   [B, Hkv, R, D]
* INT4 middle, bit-packed            mid_kq/vq  [B, Hkv, cap, D/2] u8,
  K per-channel scale [B, Hkv, 1, D], V per-token scale [B, Hkv, cap, 1],
  valid length mid_len [B] (int32, on the device).

One decode step of one layer is one C-ABI call, ``fade_decode_attn_age_out``:
the oldest ring token is quantised into the middle (K against its frozen
per-channel scale, V with its own per-token scale), the new token takes its
ring slot, and the layer's query attends over sink + middle + ring straight
from the compressed tiers.  ``fused=False`` issues the same step as the two
separate calls ``fade_age_out_int4`` + ``fade_decode_attn``.
All positions live in device memory, so ``capture()`` records the whole
multi-layer step in one CUDA graph and ``replay()`` re-runs it.

Initial tiers come from a prompt through the reference-exact quantisers
(``quant_k_int4`` / ``quant_v_int4`` over the middle, fade/quant.py:61-92).
The per-step age-out is an extension: the reference keeps new tokens in FP16
until its next full reassignment (fade/cache.py:881-1057).
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from fade_b200 import _lib
from fade_b200.attention import DecodePlan, FPTier, Int4Tier
from fade_b200.quant import quant_k_int4, quant_v_int4


def age_out_int4(ring_k: Tensor, ring_v: Tensor, mid_kq: Tensor, mid_vq: Tensor, mid_vs: Tensor,
                 k_scale: Tensor, mid_len: Tensor, ring_origin: int = 0,
                 k_new: Tensor | None = None, v_new: Tensor | None = None) -> None:
    """Move the oldest ring token of every (b, h) into the INT4 middle (see
    ``fade_age_out_int4`` in include/fade_b200.h) and put ``k_new``/``v_new``
    ([B, H, D]) in the freed slot.  ``mid_len`` (int32 [B], device) advances."""
    dev = _lib.require_cuda(ring_k, ring_v, mid_kq, mid_vq, mid_vs, k_scale, mid_len)
    B, H, R, D = ring_k.shape
    if ring_k.stride() != ring_v.stride() or ring_k.stride(3) != 1 or ring_k.stride(2) != D:
        raise ValueError("ring_k / ring_v must share a row-contiguous layout")
    rbk = D // 2
    if mid_kq.stride(3) != 1 or mid_kq.stride(2) != rbk or mid_kq.stride() != mid_vq.stride():
        raise ValueError("middle codes must be row-contiguous and share a layout")
    mid_sb, mid_sh = mid_kq.stride(0) // rbk, mid_kq.stride(1) // rbk
    if mid_vs.stride(0) != mid_sb or mid_vs.stride(1) != mid_sh or mid_vs.stride(2) != 1:
        raise ValueError("v scales must be indexed like the code rows")
    ks = k_scale.reshape(B, H, D)
    if not ks.is_contiguous():
        raise ValueError("k_scale must be contiguous")
    if mid_len.dtype != torch.int32 or mid_len.numel() != B:
        raise ValueError("mid_len must be int32 [B]")
    new_sb = new_sh = 0
    if k_new is not None:
        if k_new.shape != (B, H, D) or v_new is None or v_new.stride() != k_new.stride() or k_new.stride(2) != 1:
            raise ValueError("k_new / v_new must be [B, H, D] with a shared layout")
        new_sb, new_sh = k_new.stride(0), k_new.stride(1)
    st = _lib.bind(dev)
    _lib.check(
        _lib.load().fade_age_out_int4(
            ring_k.data_ptr(), ring_v.data_ptr(), _lib.dtype_code(ring_k.dtype), B, H, D, R,
            ring_k.stride(0), ring_k.stride(1), int(ring_origin), mid_kq.data_ptr(), mid_vq.data_ptr(),
            mid_vs.data_ptr(), ks.data_ptr(), mid_sb, mid_sh, mid_kq.shape[2], mid_len.data_ptr(),
            _lib.ptr(k_new), _lib.ptr(v_new), new_sb, new_sh, st,
        ),
        "age_out_int4",
    )


class _Layer:
    __slots__ = ("sink_k", "sink_v", "ring_k", "ring_v", "mid_kq", "mid_ks", "mid_vq", "mid_vs",
                 "mid_len", "ring_origin", "plan", "age_args", "age_desc")


class TieredDecoder:
    """Batched multi-layer decode over FADE tiers with fused sm_100a kernels.

    Args:
        n_layers, batch, n_q_heads, n_kv_heads, head_dim, dtype: model shape.
        n_sink, recent_window: FP tiers (FadeConfig.safe(): 4 and 64).
        mid_capacity: INT4 middle capacity per (b, h) in tokens (prompt middle
            plus the tokens decoding will age out).
    """

    def __init__(self, n_layers: int, batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.bfloat16, n_sink: int = 4, recent_window: int = 64,
                 mid_capacity: int = 8192, device: torch.device | str = "cuda", sm_scale: float | None = None,
                 fused: bool = True, n_ctas: int = 0):
        self.L, self.B, self.Hq, self.Hkv, self.D = n_layers, batch, n_q_heads, n_kv_heads, head_dim
        self.dtype, self.n_sink, self.R = dtype, n_sink, recent_window
        self.cap = int(-(-mid_capacity // 128) * 128)
        self.device = torch.device(device)
        self.sm_scale = sm_scale
        self.fused = fused
        # middle-kernel CTAs (0 = one per SM); fewer leaves SMs free for work
        # that should overlap the layers, e.g. collectives on another stream
        self.n_ctas = int(n_ctas)
        B, H, D = batch, n_kv_heads, head_dim
        dev = self.device
        self.q = torch.zeros(n_layers, B, n_q_heads, 1, D, dtype=dtype, device=dev)
        self.k_new = torch.zeros(n_layers, B, H, D, dtype=dtype, device=dev)
        self.v_new = torch.zeros(n_layers, B, H, D, dtype=dtype, device=dev)
        self.out = torch.zeros(n_layers, B, n_q_heads, 1, D, dtype=dtype, device=dev)
        self.layers: list[_Layer] = []
        for _ in range(n_layers):
            ly = _Layer()
            ly.sink_k = torch.zeros(B, H, n_sink, D, dtype=dtype, device=dev)
            ly.sink_v = torch.zeros_like(ly.sink_k)
            ly.ring_k = torch.zeros(B, H, recent_window, D, dtype=dtype, device=dev)
            ly.ring_v = torch.zeros_like(ly.ring_k)
            ly.mid_kq = torch.zeros(B, H, self.cap, D // 2, dtype=torch.uint8, device=dev)
            ly.mid_vq = torch.zeros_like(ly.mid_kq)
            ly.mid_ks = torch.zeros(B, H, 1, D, dtype=dtype, device=dev)
            ly.mid_vs = torch.zeros(B, H, self.cap, 1, dtype=dtype, device=dev)
            ly.mid_len = torch.zeros(B, dtype=torch.int32, device=dev)
            ly.ring_origin = 0
            ly.plan = None
            self.layers.append(ly)
        self._ws = None
        self._graph = None
        self._host_graph = None   # step_host's graph and the host buffers it was made for
        self._host_key = None
        self._age_fn = None

    # ------------------------------------------------------------------ set-up
    def load_prompt(self, layer: int, k: Tensor, v: Tensor) -> None:
        """Build the tiers of `layer` from prompt K (post-RoPE) / V [B, Hkv, S, D]:
        sinks = first n_sink, ring = last R tokens, middle = the rest quantised
        with the reference's INT4 quantisers."""
        ly = self.layers[layer]
        B, H, S, D = k.shape
        if S < self.n_sink + self.R:
            raise ValueError(f"prompt of {S} tokens is shorter than n_sink + recent_window")
        n_mid = S - self.n_sink - self.R
        if n_mid > self.cap:
            raise ValueError(f"middle of {n_mid} tokens exceeds mid_capacity {self.cap}")
        ly.sink_k.copy_(k[:, :, : self.n_sink])
        ly.sink_v.copy_(v[:, :, : self.n_sink])
        ly.ring_k.copy_(k[:, :, S - self.R:])
        ly.ring_v.copy_(v[:, :, S - self.R:])
        if n_mid > 0:
            kp, ks = quant_k_int4(k[:, :, self.n_sink: S - self.R])
            vp, vs = quant_v_int4(v[:, :, self.n_sink: S - self.R])
            ly.mid_kq[:, :, :n_mid].copy_(kp)
            ly.mid_vq[:, :, :n_mid].copy_(vp)
            ly.mid_vs[:, :, :n_mid].copy_(vs)
            ly.mid_ks.copy_(ks)
        ly.mid_len.fill_(n_mid)
        # ring slot j holds token S-R+j: the oldest sits at slot 0 when mid_len == n_mid
        ly.ring_origin = n_mid
        ly.plan = None
        self._graph = None
        self._host_graph = None

    def load_tiers(self, layer: int, sink_k, sink_v, ring_k, ring_v, mid_kq, mid_ks, mid_vq, mid_vs, n_mid: int,
                   ring_origin: int | None = None) -> None:
        """Install already-quantised tiers (e.g. synthetic benchmark state)."""
        ly = self.layers[layer]
        ly.sink_k.copy_(sink_k)
        ly.sink_v.copy_(sink_v)
        ly.ring_k.copy_(ring_k)
        ly.ring_v.copy_(ring_v)
        ly.mid_kq[:, :, :n_mid].copy_(mid_kq[:, :, :n_mid])
        ly.mid_vq[:, :, :n_mid].copy_(mid_vq[:, :, :n_mid])
        ly.mid_vs[:, :, :n_mid].copy_(mid_vs[:, :, :n_mid])
        ly.mid_ks.copy_(mid_ks)
        ly.mid_len.fill_(n_mid)
        ly.ring_origin = n_mid if ring_origin is None else ring_origin
        ly.plan = None
        self._graph = None
        self._host_graph = None

    def _plan(self, layer: int) -> DecodePlan:
        ly = self.layers[layer]
        if ly.plan is None:
            tiers = [
                FPTier(ly.sink_k, ly.sink_v),
                Int4Tier(ly.mid_kq, ly.mid_ks, ly.mid_vq, ly.mid_vs, lens=ly.mid_len, max_len=self.cap),
                FPTier(ly.ring_k, ly.ring_v),
            ]
            ly.plan = DecodePlan(self.q[layer], tiers, out=self.out[layer], sm_scale=self.sm_scale,
                                 workspace=self._ws, n_ctas=self.n_ctas)
            self._ws = ly.plan.workspace
            # prebuilt argument tuple for fade_age_out_int4 (no per-step Python work)
            B, H, R, D = ly.ring_k.shape
            rbk = D // 2
            kn, vn = self.k_new[layer], self.v_new[layer]
            ly.age_args = (
                ly.ring_k.data_ptr(), ly.ring_v.data_ptr(), _lib.dtype_code(self.dtype), B, H, D, R,
                ly.ring_k.stride(0), ly.ring_k.stride(1), int(ly.ring_origin), ly.mid_kq.data_ptr(),
                ly.mid_vq.data_ptr(), ly.mid_vs.data_ptr(), ly.mid_ks.data_ptr(), ly.mid_kq.stride(0) // rbk,
                ly.mid_kq.stride(1) // rbk, self.cap, ly.mid_len.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                kn.stride(0), kn.stride(1),
            )
            a = _lib.AgeOutDesc()
            a.ring_seg, a.mid_seg = 2, 1
            a.ring_cap, a.ring_origin = R, int(ly.ring_origin)
            a.k_new, a.v_new = kn.data_ptr(), vn.data_ptr()
            a.new_sb, a.new_sh = kn.stride(0), kn.stride(1)
            # With two or more layers the kernel preceding a layer's call is
            # another layer's, which never writes this layer's tiers or their
            # lengths, so the middle may stream early.  With one layer it is
            # this layer's previous call, whose finisher advances the lengths.
            a.prefetch_tiers = 1 if len(self.layers) > 1 else 0
            ly.age_desc = a
        return ly.plan

    # ------------------------------------------------------------------- step
    def _launch_all(self, layer_events: list | None = None, before=None, after=None) -> None:
        lib = _lib.load()
        st = _lib.bind(self.device)
        for i, ly in enumerate(self.layers):
            if before is not None:
                before(i)
            p = self._plan(i)
            if self.fused:
                if layer_events is not None:
                    layer_events[i][0].record()
                _lib.check(lib.fade_decode_attn_age_out(ctypes.byref(p.desc), ctypes.byref(ly.age_desc),
                                                        p.workspace.data_ptr(), p.ws_bytes, st),
                           "fade_decode_attn_age_out")
            else:
                _lib.check(lib.fade_age_out_int4(*ly.age_args, st), "age_out_int4")
                if layer_events is not None:
                    layer_events[i][0].record()
                _lib.check(lib.fade_decode_attn(ctypes.byref(p.desc), p.workspace.data_ptr(), p.ws_bytes, st),
                           "fade_decode_attn")
            if layer_events is not None:
                layer_events[i][1].record()
            if after is not None:
                after(i)

    def step(self, q: Tensor | None = None, k_new: Tensor | None = None, v_new: Tensor | None = None,
             after=None) -> Tensor:
        """One decode step over all layers.  q [L,B,Hq,1,D], k_new/v_new [L,B,Hkv,D]
        (copied into the static input buffers when given).  Returns the static
        output buffer [L,B,Hq,1,D]."""
        if q is not None:
            self.q.copy_(q, non_blocking=True)
        if k_new is not None:
            self.k_new.copy_(k_new, non_blocking=True)
            self.v_new.copy_(v_new, non_blocking=True)
        if self._graph is not None and after is None:
            self._graph.replay()
        else:
            self._launch_all(after=after)
        return self.out

    def capture(self, layer_events: list | None = None, after=None) -> torch.cuda.CUDAGraph:
        """Record one full step (every layer's age-out + attention) as a CUDA graph.
        Call after a warm-up step; replays then advance the cache like step().
        `layer_events` (pairs of ``torch.cuda.Event(enable_timing=True,
        external=True)``) bracket each layer's attention call inside the graph.
        `after(i)` is called after layer i's launch on the capture stream (e.g.
        a collective over that layer's output); it is recorded into the graph."""
        for i in range(self.L):
            self._plan(i)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._launch_all(layer_events, after=after)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        if layer_events is None and after is None:
            self._graph = g
        return g

    def step_host(self, q_host: Tensor, k_host: Tensor, v_host: Tensor, out_host: Tensor) -> Tensor:
        """End-to-end step from host buffers: H2D of the step's inputs (q
        [L,B,Hq,1,D], new K/V [L,B,Hkv,D]; pinned memory for async copies),
        the step itself, D2H of the attention outputs into ``out_host``.  All
        on the current stream; the caller synchronises before reading."""
        key = (q_host.data_ptr(), k_host.data_ptr(), v_host.data_ptr(), out_host.data_ptr())
        if self._host_graph is not None and self._host_key == key:
            self._host_graph.replay()
            return out_host
        self.q.copy_(q_host, non_blocking=True)
        self.k_new.copy_(k_host, non_blocking=True)
        self.v_new.copy_(v_host, non_blocking=True)
        if self._graph is not None:
            self._graph.replay()
        else:
            self._launch_all()
        out_host.copy_(self.out, non_blocking=True)
        return out_host

    def capture_host(self, q_host: Tensor, k_host: Tensor, v_host: Tensor, out_host: Tensor) -> torch.cuda.CUDAGraph:
        """Record step_host for these (pinned) host buffers as one CUDA graph in
        which the copies overlap the layers.  A side stream copies the inputs
        in layer chunks of growing size (1, 3, 12, 48, ... layers: the first
        layer starts after one layer's copies, and each later chunk lands long
        before its first layer runs, since a layer's copies take a fraction of
        its attention time); the layers wait only at chunk boundaries, so the
        kernels of consecutive layers keep their programmatic dependent
        launches everywhere else.  Outputs go back in the mirrored chunks (the
        last layer's alone).  Later step_host calls with the same buffers
        replay it.  Call after a warm-up step."""
        for i in range(self.L):
            self._plan(i)
        dev = self.device
        L = self.L
        sizes, n = [], 1
        while sum(sizes) < L:
            sizes.append(min(n, L - sum(sizes)))
            n = 3 if n == 1 else 4 * n
        in_chunks, a = [], 0
        for z in sizes:
            in_chunks.append((a, a + z))
            a += z
        out_chunks, a = [], 0
        for z in reversed(sizes):
            out_chunks.append((a, a + z))
            a += z
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        s, cin, cout = (torch.cuda.Stream(dev) for _ in range(3))
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                start = torch.cuda.Event()
                start.record(s)
                cin.wait_event(start)
                cout.wait_event(start)
                ev_in = {}
                with torch.cuda.stream(cin):
                    for i0, i1 in in_chunks:
                        self.q[i0:i1].copy_(q_host[i0:i1], non_blocking=True)
                        self.k_new[i0:i1].copy_(k_host[i0:i1], non_blocking=True)
                        self.v_new[i0:i1].copy_(v_host[i0:i1], non_blocking=True)
                        e = torch.cuda.Event()
                        e.record(cin)
                        ev_in[i0] = e
                out_last = {i1 - 1: i0 for i0, i1 in out_chunks}

                def before(i):
                    if i in ev_in:
                        s.wait_event(ev_in[i])

                def after(i):
                    if i not in out_last:
                        return
                    i0 = out_last[i]
                    e = torch.cuda.Event()
                    e.record(s)
                    cout.wait_event(e)
                    with torch.cuda.stream(cout):
                        out_host[i0:i + 1].copy_(self.out[i0:i + 1], non_blocking=True)

                self._launch_all(before=before, after=after)
                s.wait_stream(cin)
                s.wait_stream(cout)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self._host_graph = g
        self._host_key = (q_host.data_ptr(), k_host.data_ptr(), v_host.data_ptr(), out_host.data_ptr())
        return g

    def replay(self) -> None:
        if self._graph is None:
            raise RuntimeError("capture() first")
        self._graph.replay()

    def check_device_errors(self) -> None:
        if self.layers and self.layers[0].plan is not None:
            self.layers[0].plan.check_device_errors()

    # --------------------------------------------------------------- metrics
    def mid_lengths(self) -> list[int]:
        return [int(ly.mid_len[0]) for ly in self.layers]

    def step_bytes(self, n_mid: int | None = None) -> int:
        """Algorithmic HBM bytes of one step: every compressed tier read once
        (codes + scales), q read, out written, plus the age-out (one FP token
        read, its INT4 row and scale written, the new token read and written)."""
        eb = torch.tensor([], dtype=self.dtype).element_size()
        Z = self.B * self.Hkv
        g = self.Hq // self.Hkv
        D = self.D
        total = 0
        for ly in self.layers:
            n = int(ly.mid_len[0]) if n_mid is None else n_mid
            per_z = (self.n_sink + self.R) * D * 2 * eb + n * (D + eb) + D * eb + 2 * g * D * eb
            age = 2 * D * eb + D + eb + 2 * (2 * D * eb)
            total += Z * (per_z + age)
        return total
