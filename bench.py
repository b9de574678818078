"""Benchmark: FADE tiered decode attention on B200.

Configurations (``--config``, default 2; synthetic seeded data of each
configuration's shape, N(0,1) K/V with 4 outlier channels per head x8):
  1  Qwen2.5-0.5B shape, 1 layer, batch 1, 14/2 heads, head_dim 64, fp16,
     context 2048 = 4 sink + 64 recent FP + 1980 INT4 middle.
  2  Llama-3.1-8B shape, 32 layers, batch 16, 32/8 heads, head_dim 128, bf16,
     context 8192 = 4 + 64 FP + 8124 INT4 middle (the headline).
  3  Mistral-7B shape H2O, 32 layers, batch 8, 32/8 heads, fp16: a 4096-token
     prompt compacted to 4 + 64 FP + 400 survivors (K INT4, V INT2 group 32),
     re-RoPE'd at contiguous positions; decode over the compacted cache.
  4  Qwen2.5-7B shape, 28 layers, 64 ragged sequences (512..32768 tokens),
     28/4 heads, bf16, rotated 2-bit middle, per-sequence tier boundaries.
  5  Llama-3-70B shape, 80 layers, 64/8 heads, bf16, context 32768 = 4 + 128
     FP + 32636 INT4 middle; batch 16 per GPU-equivalent (128 at 8 GPUs).
Configurations 1, 2 and 5 run one decode step per layer as
``fade_decode_attn_age_out`` (the token leaving the recent window is
quantised into the middle, then the fused attention), replayed as a CUDA
graph.

Multi-GPU (torchrun, one process per GPU; configs 2 and 5): weak scaling with
the batch growing with N.  Default partition "heads": rank r holds kv heads
[r*Hkv/N, (r+1)*Hkv/N) of the whole batch (one kv head per GPU at N=8) and
every layer's attention output is all-gathered over NCCL inside the timed
step; "--shard batch" gives each rank its own batch slice with no collective.
The step time is the max over ranks; the value is the whole job's throughput.

Usage: python bench.py [--config C] [--gpus N] [--steps K] [--warmup W] [--impl fade|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    1: dict(kind="int4", layers=1, batch=1, n_q_heads=14, n_kv_heads=2, head_dim=64, context=2048, n_sink=4,
            recent=64, dtype="f16", theta=1e6,
            workload="config 1: Qwen2.5-0.5B-shaped single-layer tiered decode (4 sink + 64 recent FP, 1980 INT4)",
            metric="tiered decode-attn effective KV GB/s (Qwen2.5-0.5B shape, 1 layer, step incl. age-out)"),
    2: dict(kind="int4", layers=32, batch=16, n_q_heads=32, n_kv_heads=8, head_dim=128, context=8192, n_sink=4,
            recent=64, dtype="bf16", theta=5e5,
            workload="config 2: Llama-3.1-8B-shaped tiered decode (4 sink + 64 recent FP, 8124 INT4 middle)",
            metric="tiered decode-attn effective KV GB/s (Llama-3.1-8B shape, 32 layers, step incl. age-out)"),
    3: dict(kind="h2o", layers=32, batch=8, n_q_heads=32, n_kv_heads=8, head_dim=128, prompt=4096, n_sink=4,
            recent=64, budget=400, group=32, dtype="f16", theta=1e6,
            workload="config 3: Mistral-7B-shaped H2O decode over the compacted cache (4096 -> 4 + 64 FP "
                     "+ 400 INT4-K / INT2-V g32 survivors, re-RoPE'd)",
            metric="tiered decode-attn effective KV GB/s (Mistral-7B shape H2O, 32 layers)"),
    4: dict(kind="rot", layers=28, n_seq=64, n_q_heads=28, n_kv_heads=4, head_dim=128, lo=512, hi=32768,
            n_sink=4, recent=64, bits=2, dtype="bf16",
            workload="config 4: Qwen2.5-7B-shaped ragged batch (64 sequences, 512..32768 tokens), rotated "
                     "2-bit middle",
            metric="tiered decode-attn effective KV GB/s (Qwen2.5-7B shape ragged rotated 2-bit, 28 layers)"),
    5: dict(kind="int4", layers=80, batch=16, n_q_heads=64, n_kv_heads=8, head_dim=128, context=32768, n_sink=4,
            recent=128, dtype="bf16", theta=5e5,
            workload="config 5: Llama-3-70B-shaped tiered decode (4 sink + 128 recent FP, 32636 INT4 middle)",
            metric="tiered decode-attn effective KV GB/s (Llama-3-70B shape, 80 layers, step incl. age-out)"),
}
L2_BYTES = 126 * 1024 * 1024
CFG: dict = {}
# default timed steps per configuration (about 1 s of device time on one B200;
# configurations 1 and 3 flush L2 between steps, outside the timed events)
DEFAULT_STEPS = {1: 2000, 2: 700, 3: 1000, 4: 250, 5: 90}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: about 1 s of timed work for the configuration)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("fade", "reference"), default="fade")
    ap.add_argument("--shard", choices=("heads", "batch"), default=None,
                    help="multi-GPU partition (default: heads)")
    ap.add_argument("--eager", action="store_true", help="launch the step eagerly (no CUDA graph)")
    ap.add_argument("--gather-stream", choices=("inline", "side"), default="side",
                    help="multi-GPU heads partition: all-gather each layer on the compute stream, or on a side "
                         "stream overlapping the next layers")
    ap.add_argument("--reassign", action="store_true",
                    help="time the tier-reassignment kernels (quantisers, rotation, re-RoPE, dequant) instead")
    ap.add_argument("--reserve-sms", type=int, default=None,
                    help="multi-GPU heads partition with side-stream gathers: SMs left free of the persistent "
                         "middle kernel for the collective (default 0: at 8 GPUs, config 2, 8 reserved SMs "
                         "measured 1.668 vs 1.645 ms/step with none)")
    ap.add_argument("--middle", choices=("mma_sync", "tcgen05"), default="mma_sync",
                    help="middle kernel for INT4 K and V at head_dim 128 (configs 2 and 5)")
    ap.add_argument("--hf", action="store_true",
                    help="time a Hugging Face decode step (random-init Llama-3.1-8B-shaped model, config 2's "
                         "batch and context) through create_tiered_cache: fused attention vs materialise + SDPA")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=None, help="layers per step (profiling captures use 1)")
    ap.add_argument("--batch", type=int, default=None, help="batch per GPU-equivalent (default: the config's)")
    args = ap.parse_args()
    if args.steps is None:   # roughly one second of timed steps, so clock samples cover the load
        args.steps = 10 if args.impl == "reference" else (
            DEFAULT_STEPS[args.config] if not (args.reassign or args.hf) else 50)
    CFG.update(CONFIGS[args.config])
    CFG["id"] = args.config
    if args.layers:
        CFG["layers"] = args.layers
    if args.batch:
        CFG["batch"] = args.batch
    CFG["middle"] = args.middle
    return args


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _eb() -> int:
    return 2


def int4_bytes(n_mid: int, Z: int, g: int, cfg=CFG) -> tuple[int, int]:
    """(decode-attention bytes of one layer, age-out bytes of one layer) for Z
    (b, kv-head) rows.  Per row: FP tiers K+V, INT4 K and V codes (D/2 B each
    per token), per-token V scale, per-channel K scale, q read + out written
    for its g heads.  Age-out: one FP token read, its INT4 row + scale
    written, the new token read and written into the ring."""
    D, eb = cfg["head_dim"], _eb()
    fp = (cfg["n_sink"] + cfg["recent"]) * D * 2 * eb
    per_z = fp + n_mid * (D + eb) + D * eb + 2 * g * D * eb
    age = 2 * D * eb + D + eb + 2 * (2 * D * eb)
    return Z * per_z, Z * age


# --------------------------------------------------------------------------
# clocks sampling during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids):
        # torch reports the PCI bus number as an int; nvidia-smi as "dddddddd:bb:dd.f"
        self.bus_ids = {int(b) for b in bus_ids if b is not None}
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        rows = [r.split(",") for r in Path(self.tmp.name).read_text().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        mine = []
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 10:
                continue
            try:
                bus = int(r[1].split(":")[1], 16)
            except (IndexError, ValueError):
                continue
            if bus in self.bus_ids:
                mine.append(r)
        if not mine:
            mine = [[x.strip() for x in r] for r in rows if len(r) >= 10]
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in mine if r[3].replace(".", "").isdigit()]
        load = [x for x in sm if mx and x > 0.5 * max(mx)] or sm
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in mine:
            for name, val in zip(names, r[6:10]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mine)}


# --------------------------------------------------------------------------
# host description and the reference's CPU path
# --------------------------------------------------------------------------
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def host_cpu() -> dict:
    model, cores = None, set()
    try:
        phys = core = None
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "model name" and model is None:
                model = v
            elif k == "physical id":
                phys = v
            elif k == "core id":
                core = v
                cores.add((phys, core))
    except Exception:
        pass
    return {"cpu_model": model, "physical_cores": len(cores) or None, "threads_available": cpu_threads()}


def _reference_modules():
    """The reference installed under baseline/_ref (its own stock code); None
    when absent, in which case the CPU numbers come from the oracle's
    restatement of the same per-step path."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "fade").is_dir():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        import fade.cache
        import fade.policy
        import fade.rotated_quant
        return fade
    except Exception:
        return None


def _torch_dt(name):
    import torch
    return {"bf16": torch.bfloat16, "f16": torch.float16}[name]


def time_reference_int4(B: int, Hkv: int, Hq: int, S: int, steps: int, warmup: int, threads: int):
    """Seconds per single-layer decode step of the reference on the CPU:
    TieredKVCache.update(new token) -- which returns the materialised
    cat(sink, cached dequant middle, recent) (fade/cache.py:347-401, 693-808)
    -- then scaled_dot_product_attention(enable_gqa) as HF's SDPA module does.
    Returns (samples, kind)."""
    import torch
    import torch.nn.functional as F

    torch.set_num_threads(threads)
    dt = _torch_dt(CFG["dtype"])
    D, ns, nr = CFG["head_dim"], CFG["n_sink"], CFG["recent"]
    gen = torch.Generator().manual_seed(0)
    fade = _reference_modules()
    q = torch.randn(B, Hq, 1, D, generator=gen).to(dt)
    if fade is None:
        from oracle.cpu_path import time_layer_steps
        return time_layer_steps(B, Hq, Hkv, D, ns, S - ns - nr, nr, dt, steps, warmup, threads), "port"
    k = torch.randn(B, Hkv, S, D, generator=gen).to(dt)
    v = torch.randn(B, Hkv, S, D, generator=gen).to(dt)
    cache = fade.cache.TieredKVCache(n_sink=ns, recent_window=nr, int4_budget=None, dtype=dt, head_dim=D,
                                     rope_theta=CFG.get("theta", 1e4))
    cache.update(k, v, 0)
    cache.apply_tier_assignment(0, fade.policy._assign_one_layer(S, torch.arange(S, dtype=torch.float32), ns, nr,
                                                                 None, 0))
    del k, v
    out = []
    for i in range(warmup + steps):
        kn = torch.randn(B, Hkv, 1, D, generator=gen).to(dt)
        vn = torch.randn(B, Hkv, 1, D, generator=gen).to(dt)
        t0 = time.perf_counter()
        K, V = cache.update(kn, vn, 0)
        F.scaled_dot_product_attention(q, K, V, enable_gqa=True)
        if i >= warmup:
            out.append(time.perf_counter() - t0)
    return out, "reference"


def reference_step_seconds(steps: int, warmup: int, threads: int, rows_total: int):
    """(seconds per full step, kind, sample text) of the reference's CPU path
    for the configuration, from a bounded sample scaled to the whole step."""
    c = CFG
    L = c["layers"]
    if c["id"] == 5:
        # one sequence (8 kv heads) of one layer, scaled by bytes: the full
        # configuration's compressed state does not fit a host
        samples, kind = time_reference_int4(1, c["n_kv_heads"], c["n_q_heads"], c["context"], steps, warmup,
                                            threads)
        scale = rows_total / c["n_kv_heads"] * L
        what = (f"1 sequence x 1 layer timed per step, scaled x{scale:g} by rows and layers (extrapolated): "
                f"reference TieredKVCache.update + SDPA on the CPU, context {c['context']}")
    else:
        B = rows_total // c["n_kv_heads"]
        samples, kind = time_reference_int4(B, c["n_kv_heads"], c["n_q_heads"], c["context"], steps, warmup,
                                            threads)
        scale = L
        what = (f"1 of {L} layers timed per step, x{L} (extrapolated over layers): reference "
                f"TieredKVCache.update + SDPA(enable_gqa) on the CPU, batch {B}, context {c['context']}")
    if kind == "port":
        what += " [oracle restatement: the reference is not installed]"
    return statistics.mean(samples) * scale, kind, what


def run_reference(args, ws, rank):
    if rank != 0:
        return
    if CFG["kind"] != "int4":
        print(json.dumps({"impl": "reference", "unavailable": f"reference arm is implemented for configs 1, 2 "
                                                              f"and 5 (config {CFG['id']} requested)"}))
        return
    threads = cpu_threads()
    steps = max(1, args.steps)
    rows = CFG["batch"] * ws * CFG["n_kv_heads"]
    t, kind, sample = reference_step_seconds(steps, max(1, min(args.warmup, 3)), threads, rows)
    n_mid = CFG["context"] - CFG["n_sink"] - CFG["recent"]
    g = CFG["n_q_heads"] // CFG["n_kv_heads"]
    dec_b, _ = int4_bytes(n_mid, rows, g)
    val = dec_b * CFG["layers"] / t / 1e9
    line = {
        "impl": "reference", "metric": CFG["metric"], "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": CFG["dtype"],
        "data": "synthetic", "config": config_block(ws, "reference (CPU)"),
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample,
                         **host_cpu()},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(ws: int, parallelism: str) -> dict:
    c = CFG
    blk = {"workload": c["workload"], "layers": c["layers"], "n_q_heads": c["n_q_heads"],
           "n_kv_heads": c["n_kv_heads"], "head_dim": c["head_dim"], "parallelism": parallelism}
    if c["kind"] == "int4":
        blk.update(batch_per_gpu=c["batch"], global_batch=c["batch"] * ws, context=c["context"],
                   n_sink=c["n_sink"], recent=c["recent"], middle_kernel=c.get("middle", "mma_sync"))
    return blk


# --------------------------------------------------------------------------
# fade arm: configs 1, 2, 5 (TieredDecoder: age-out + fused attention per layer)
# --------------------------------------------------------------------------
def build_decoder(dev, extra_steps, plan, seed_base, n_ctas=0):
    import torch

    from fade_b200.decoder import TieredDecoder

    c = CFG
    dt = _torch_dt(c["dtype"])
    n_mid = c["context"] - c["n_sink"] - c["recent"]
    dec = TieredDecoder(c["layers"], plan.batch, plan.n_q_heads, plan.n_kv_heads, c["head_dim"], dtype=dt,
                        n_sink=c["n_sink"], recent_window=c["recent"], mid_capacity=n_mid + extra_steps + 8,
                        device=dev, n_ctas=n_ctas)
    gen = torch.Generator(device=dev)
    B, H, S, D = plan.batch, plan.n_kv_heads, c["context"], c["head_dim"]
    for layer in range(c["layers"]):
        gen.manual_seed(seed_base + layer)
        k = torch.randn(B, H, S, D, device=dev, generator=gen)
        v = torch.randn(B, H, S, D, device=dev, generator=gen)
        for h in range(H):
            ch = torch.randperm(D, device=dev, generator=gen)[:4]
            k[:, h, :, ch] *= 8.0
            v[:, h, :, ch] *= 8.0
        dec.load_prompt(layer, k.to(dt), v.to(dt))
        del k, v
    torch.cuda.synchronize(dev)
    return dec, n_mid


def _measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def run_int4(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from fade_b200.attention import set_middle_kernel
    from fade_b200.shard import gather_objects, max_over_ranks, shard_plan

    c = CFG
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    set_middle_kernel(c["middle"])
    K, W = args.steps, max(3, args.warmup)
    L = c["layers"]
    mode = args.shard or "heads"
    plan = shard_plan(mode if ws > 1 else "batch", ws, rank, c["batch"] * ws, c["n_q_heads"], c["n_kv_heads"])
    g = c["n_q_heads"] // c["n_kv_heads"]
    Z = plan.batch * plan.n_kv_heads
    n_mid0 = c["context"] - c["n_sink"] - c["recent"]
    step_bytes0 = sum(int4_bytes(n_mid0, Z, g)) * L
    small = step_bytes0 < 2 * L2_BYTES              # fits in L2: flush between timed steps
    roof_steps = min(K, 10) if ws == 1 else 0
    e2e_steps = 0 if args.no_e2e else min(K, 20)
    total = 4 + 2 * W + 3 * K + roof_steps + e2e_steps
    n_ctas = 0
    if plan.gathers and args.gather_stream == "side":
        reserve = 0 if args.reserve_sms is None else max(0, args.reserve_sms)
        n_ctas = max(1, torch.cuda.get_device_properties(dev).multi_processor_count - reserve)
    dec, _ = build_decoder(dev, total, plan, 1000 + 100003 * rank, n_ctas=n_ctas)
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    dt = _torch_dt(c["dtype"])
    q = torch.randn(dec.q.shape, device=dev, generator=gen).to(dt)
    kn = torch.randn(dec.k_new.shape, device=dev, generator=gen).to(dt)
    vn = torch.randn(dec.v_new.shape, device=dev, generator=gen).to(dt)

    after, gathered = None, None
    if plan.gathers:
        # every layer's output [B, Hq/N, 1, D] is all-gathered into [N, B, Hq/N, 1, D]
        gathered = torch.empty((L, ws) + tuple(dec.out.shape[1:]), dtype=dt, device=dev)

        side = torch.cuda.Stream(dev)

        def after_inline(i):
            dist.all_gather_into_tensor(gathered[i], dec.out[i])

        def after_side(i):
            # layer i's gather overlaps layers i+1..; the step ends when every gather has
            cur = torch.cuda.current_stream(dev)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                dist.all_gather_into_tensor(gathered[i], dec.out[i])
            if i == L - 1:
                cur.wait_stream(side)

        after = after_inline if args.gather_stream == "inline" else after_side

    dec.step(q, kn, vn, after=after)          # eager step: builds plans, warms the communicator
    torch.cuda.synchronize(dev)
    graph_ok = not args.eager
    try:
        if args.eager:
            raise RuntimeError("--eager")
        g_main = dec.capture(after=after)
    except Exception as e:                     # NCCL capture unsupported: eager steps
        graph_ok, g_main = False, None
        print(f"[bench] graph capture with the collective failed ({type(e).__name__}: {e}); eager steps",
              file=sys.stderr)
        torch.cuda.synchronize(dev)

    def one_step():
        if g_main is not None:
            g_main.replay()
        else:
            dec.step(after=after)

    for _ in range(W):
        one_step()
    torch.cuda.synchronize(dev)
    dec.check_device_errors()
    n_mid_start = n_mid0 + 1 + W

    props = torch.cuda.get_device_properties(dev)
    bus_ids = [b for b in gather_objects(getattr(props, "pci_bus_id", None)) if b is not None]
    sampler = ClockSampler(bus_ids) if rank == 0 else None

    # ---------------- timed region: K steps ----------------
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if small else None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:                 # before the barrier: no rank may wait for it inside the timed region
        sampler.start()
        time.sleep(0.3)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record()
    for i in range(K):
        if small:
            flush.zero_()                      # L2 flushed outside each step's events
            evs[i][0].record()
            one_step()
            evs[i][1].record()
        else:
            one_step()
    e1.record()
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_local = sum(a.elapsed_time(b) for a, b in evs) if small else e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms_local, dev)
    dec.check_device_errors()
    tot_bytes = sum(sum(int4_bytes(n_mid_start + i + 1, Z, g)) * L for i in range(K))
    step_ms = ms_max / K
    value = tot_bytes * ws / (ms_max / 1e3) / 1e9
    n_next = n_mid_start + K

    # hot-L2 steps back to back (small configurations only)
    hot = None
    if small:
        torch.cuda.synchronize(dev)
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record()
        for _ in range(K):
            one_step()
        h1.record()
        torch.cuda.synchronize(dev)
        hot = {"us_per_step": round(max_over_ranks(h0.elapsed_time(h1), dev) / K * 1e3, 2),
               "note": "inputs fit in L2; back-to-back steps, no flush (not an HBM number)"}
        n_next += K

    # collective share: the same step recorded without the all-gathers, and
    # with each gather on the compute stream (the next layer then waits for it)
    coll = None
    if plan.gathers:
        def timed_variant(hook):
            try:
                gv = dec.capture(after=hook)
                torch.cuda.synchronize(dev)
                for _ in range(2):
                    gv.replay()
                torch.cuda.synchronize(dev)
                dist.barrier()
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record()
                for _ in range(K):
                    gv.replay()
                c1.record()
                torch.cuda.synchronize(dev)
                return max_over_ranks(c0.elapsed_time(c1), dev) / K
            except Exception:
                return None

        ms_ng = timed_variant(None)
        other = after_inline if args.gather_stream == "side" else after_side
        ms_other = timed_variant(other)
        n_next += 2 * (K + 2)
        per_layer = int(dec.out[0].numel() * dec.out.element_size())
        coll = {"op": "all_gather (NCCL) of each layer's attention output", "ranks": ws,
                "stream": args.gather_stream,
                "middle_kernel_ctas": n_ctas or "one per SM",
                "bytes_in_per_rank_per_layer": per_layer, "bytes_out_per_layer": per_layer * ws,
                "graph_captured": graph_ok,
                "ms_per_step_without_collective": round(ms_ng, 4) if ms_ng else None,
                ("ms_per_step_inline" if args.gather_stream == "side" else "ms_per_step_side"):
                    round(ms_other, 4) if ms_other else None,
                "share_of_step": round(1 - ms_ng / step_ms, 4) if ms_ng else None}

    # ---------------- roofline (per GPU) ----------------
    avg_ms = step_ms / L
    attn_bytes = tot_bytes / (K * L)
    achieved = attn_bytes / (avg_ms / 1e3) / 1e9
    iso_us = None
    if roof_steps:
        lev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
               for _ in range(L)]
        g2 = dec.capture(layer_events=lev)
        durs = []
        for _ in range(roof_steps):
            g2.replay()
            torch.cuda.synchronize(dev)
            durs.extend(a.elapsed_time(b) for a, b in lev)
        iso_us = statistics.mean(durs) * 1e3
        n_next += roof_steps
    peaks = _measured_peaks()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    if c["id"] == 2:
        try:
            traffic = json.loads((ROOT / "profiles" / "decode_attn_traffic.json").read_text()).get(
                "bytes_per_launch_scaled")
        except Exception:
            pass

    # ---------------- e2e through the public API with host buffers ----------------
    e2e = None
    if e2e_steps:
        qh, kh, vh = q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory()
        oh = torch.empty(dec.out.shape, dtype=dec.out.dtype).pin_memory()
        dec.step_host(qh, kh, vh, oh)
        dec.capture_host(qh, kh, vh, oh)      # copies overlap the layers, one graph per step
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(e2e_steps):
            dec.step_host(qh, kh, vh, oh)
        s1.record()
        torch.cuda.synchronize(dev)
        e_ms = max_over_ranks(s0.elapsed_time(s1), dev)
        n_e = n_next + 2
        eb = sum(sum(int4_bytes(n_e + i + 1, Z, g)) * L for i in range(e2e_steps))
        e2e = {"value": round(eb * ws / (e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": int((qh.numel() + kh.numel() + vh.numel()) * qh.element_size()),
               "d2h_bytes_per_step": int(oh.numel() * oh.element_size()),
               "ms_per_step": round(e_ms / e2e_steps, 4),
               "path": "TieredDecoder.step_host (pinned host inputs -> fade_decode_attn_age_out per layer -> "
                       "host output), per rank"}

    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline and ws == 1:
        threads = cpu_threads()
        t, kind, sample = reference_step_seconds(3, 1, threads, Z)
        dec_b, _ = int4_bytes(n_mid0, Z, g)
        cpu = {"value": round(dec_b * L / t / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": "3 steps: " + sample, **host_cpu()}
    par = f"{plan.mode}-sharded x{ws}" + (" + NCCL all_gather of outputs per layer" if plan.gathers else "")
    line = {
        "metric": c["metric"], "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": round(step_ms, 4), "us_per_step": round(step_ms * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"int4 codes -> {c['dtype']} ({c['dtype']} MMA, f32 accumulate)", "data": "synthetic",
        "config": {**config_block(ws, par),
                   "l2": ("inputs fit in L2: L2 flushed (a 252 MB write) between timed steps, outside their events"
                          if small else f"inputs larger than L2 ({step_bytes0 / 1e9:.2f} GB per step vs 126 MB L2)")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "fade_decode_attn_age_out per layer (middle_kernel + finish_kernel), per GPU",
                     "avg_launch_us": round(avg_ms * 1e3, 2), "bytes_per_launch": int(attn_bytes),
                     "isolated_call_us": round(iso_us, 2) if iso_us else None,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "fallback"},
        "hot_l2": hot,
        "collective": coll,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 2 * L * K,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# fade arm: configs 3 and 4 (decode over fixed tiers, one DecodePlan per layer)
# --------------------------------------------------------------------------
def _timed_graph(dev, g, K: int, small: bool):
    """ms per step over K replays of graph g (L2 flushed between steps, outside
    their events, when the inputs fit in L2), plus the clocks record."""
    import torch

    sampler = ClockSampler([getattr(torch.cuda.get_device_properties(dev), "pci_bus_id", None)])
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if small else None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize(dev)
    e0.record()
    for i in range(K):
        if small:
            flush.zero_()
            evs[i][0].record()
            g.replay()
            evs[i][1].record()
        else:
            g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ms = sum(a.elapsed_time(b) for a, b in evs) if small else e0.elapsed_time(e1)
    hot = None
    if small:
        e0.record()
        for _ in range(K):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        hot = {"us_per_step": round(e0.elapsed_time(e1) / K * 1e3, 2),
               "note": "inputs fit in L2; back-to-back steps, no flush (not an HBM number)"}
    return ms / K, clocks, hot


def _capture_plans(dev, plans):
    import torch

    for p in plans:
        p.run()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for p in plans:
                p.run()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    return g


def _fixed_tier_line(args, ms, clocks, hot, layer_bytes, extra: dict, launches_per_step: int):
    c = CFG
    L, K = c["layers"], args.steps
    step_bytes = layer_bytes * L
    peaks = _measured_peaks()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = layer_bytes / (ms / L / 1e3) / 1e9
    small = step_bytes < 2 * L2_BYTES
    return {
        "metric": c["metric"], "value": round(step_bytes / (ms / 1e3) / 1e9, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": K, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4), "us_per_step": round(ms * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": c["dtype"], "data": "synthetic",
        "config": {**config_block(1, "single GPU"), **extra.pop("config", {}),
                   "l2": ("inputs fit in L2: L2 flushed (a 252 MB write) between timed steps, outside their events"
                          if small else f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step)")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "kernel": "fade_decode_attn per layer (middle_kernel + finish_kernel)",
                     "avg_launch_us": round(ms / L * 1e3, 2), "bytes_per_launch": int(layer_bytes),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "fallback"},
        "hot_l2": hot, **extra, "cpu_baseline": None, "e2e": None,
        "gpu_launches": launches_per_step * K, "clocks": clocks,
    }


def run_h2o(args):
    """Config 3: per layer, a 4096-token prompt through the cache's eviction
    path (H2O survivors from Dirichlet(0.1) scores via _assign_one_layer,
    un-RoPE / re-RoPE, K INT4 + V INT2 group 32), then the decode step over all
    layers' compacted caches as one graph."""
    import torch

    from fade_b200.attention import DecodePlan
    from fade_b200.cache import TieredKVCache
    from fade_b200.policy import _assign_one_layer, assign_counts
    from fade_b200.rope import Vanilla

    c = CFG
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, B, Hq, H, D, S = c["layers"], c["batch"], c["n_q_heads"], c["n_kv_heads"], c["head_dim"], c["prompt"]
    dt = _torch_dt(c["dtype"])
    scheme = Vanilla(theta=c["theta"], head_dim=D)
    cache = TieredKVCache(n_sink=c["n_sink"], recent_window=c["recent"], int4_budget=c["budget"], dtype=dt,
                          rope_theta=c["theta"], head_dim=D, middle_v_bits=2, rope_scheme=scheme,
                          v_int2_group_size=c["group"])
    gen = torch.Generator(device=dev).manual_seed(3)
    torch.manual_seed(3)
    reassign_ms = []
    for layer in range(L):
        k = torch.randn(B, H, S, D, device=dev, generator=gen)
        v = torch.randn(B, H, S, D, device=dev, generator=gen)
        for h in range(H):
            ch = torch.randperm(D, device=dev, generator=gen)[:4]
            k[:, h, :, ch] *= 8.0
            v[:, h, :, ch] *= 8.0
        cache.update(k.to(dt), v.to(dt), layer)
        scores = torch.distributions.Dirichlet(torch.full((S,), 0.1, device=dev)).sample((H,)).sum(0)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        args_l = (S, c["n_sink"], c["recent"], c["budget"], 0)
        cache.apply_tier_assignment(layer, _assign_one_layer(args_l[0], scores, *args_l[1:]),
                                    counts=assign_counts(*args_l))
        torch.cuda.synchronize(dev)
        reassign_ms.append((time.perf_counter() - t0) * 1e3)
        del k, v
    q = torch.randn(L, B, Hq, 1, D, device=dev, generator=gen).to(dt)
    out = torch.empty_like(q)
    plans = [DecodePlan(q[i], cache.decode_tiers(i), out=out[i]) for i in range(L)]
    g = _capture_plans(dev, plans)
    for _ in range(max(3, args.warmup)):
        g.replay()
    ms, clocks, hot = _timed_graph(dev, g, args.steps, True)
    plans[0].check_device_errors()
    n = c["budget"]
    G = c["group"]
    n_pad = -(-n // G) * G
    eb = 2
    g_ = Hq // H
    per_z = (c["n_sink"] + c["recent"]) * D * 2 * eb + n * D // 2 + D * eb + n_pad * D // 4 \
        + (n_pad // G) * D * eb + 2 * g_ * D * eb
    extra = {"reassignment": {"ms_per_layer_median": round(statistics.median(reassign_ms[1:] or reassign_ms), 3),
                              "what": "TieredKVCache.apply_tier_assignment of a 4096-token layer on the GPU "
                                      "(un-RoPE/re-RoPE gather, INT4 K + INT2 V quantisers) with the tier "
                                      "counts from the budgets (no host sync), host wall clock; not in the "
                                      "timed decode step"},
             "config": {"batch": B, "prompt": S, "int4_budget": n, "v_int2_group": G}}
    print(json.dumps(_fixed_tier_line(args, ms, clocks, hot, B * H * per_z, extra, 2 * L)), flush=True)


def run_rot(args):
    """Config 4: 64 ragged sequences (lengths uniform in [lo, hi]) in one call
    per layer: FP sink / recent tiers plus the rotated 2-bit middle in a padded
    layout read through per-sequence lengths and a ragged unit grid (only the
    real 128-token units are scheduled).  Codes and scales are random bytes of
    the right format (the quantisers are validated by the tests)."""
    import torch

    from fade_b200.attention import DecodePlan, FPTier, RotTier
    from fade_b200.rotated_quant import _random_orthogonal

    c = CFG
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, Ns, Hq, H, D = c["layers"], c["n_seq"], c["n_q_heads"], c["n_kv_heads"], c["head_dim"]
    ns, nr = c["n_sink"], c["recent"]
    dt = _torch_dt(c["dtype"])
    gcpu = torch.Generator().manual_seed(4)
    lens = torch.randint(c["lo"], c["hi"] + 1, (Ns,), generator=gcpu).tolist()
    mids = [n - ns - nr for n in lens]
    cap = -(-max(mids) // 128) * 128
    R = _random_orthogonal(D, 42).to(dev)
    lens_t = torch.tensor(mids, dtype=torch.int32, device=dev)
    units = torch.tensor([-(-m // 128) for m in mids], dtype=torch.int32).repeat_interleave(H)
    cu = torch.cat([torch.zeros(1, dtype=torch.int32), units.cumsum(0).to(torch.int32)]).to(dev)
    gen = torch.Generator(device=dev).manual_seed(5)
    rb = D * c["bits"] // 8
    plans, keep = [], []
    q = torch.randn(L, Ns, Hq, 1, D, device=dev, generator=gen).to(dt)
    out = torch.empty_like(q)
    for layer in range(L):
        kp = torch.randint(0, 256, (Ns, H, cap, rb), dtype=torch.uint8, device=dev, generator=gen)
        vp = torch.randint(0, 256, (Ns, H, cap, rb), dtype=torch.uint8, device=dev, generator=gen)
        ks = (torch.rand(Ns, H, 1, D, device=dev, generator=gen) * 2 + 0.5).to(dt)
        vs = (torch.rand(Ns, H, cap, 1, device=dev, generator=gen) * 2 + 0.5).to(dt)
        sk = torch.randn(Ns, H, ns, D, device=dev, generator=gen).to(dt)
        sv = torch.randn(Ns, H, ns, D, device=dev, generator=gen).to(dt)
        rk = torch.randn(Ns, H, nr, D, device=dev, generator=gen).to(dt)
        rv = torch.randn(Ns, H, nr, D, device=dev, generator=gen).to(dt)
        tiers = [FPTier(sk, sv), RotTier(kp, ks, vp, vs, bits=c["bits"], rotation=R, lens=lens_t, max_len=cap),
                 FPTier(rk, rv)]
        keep.append(tiers)
        plans.append(DecodePlan(q[layer], tiers, out=out[layer], cu_units=cu))
    g = _capture_plans(dev, plans)
    for _ in range(max(3, args.warmup)):
        g.replay()
    ms, clocks, hot = _timed_graph(dev, g, args.steps, False)
    plans[0].check_device_errors()
    eb, g_ = 2, Hq // H
    layer_bytes = sum(H * ((ns + nr) * D * 2 * eb + m * 2 * rb + m * eb + D * eb + 2 * g_ * D * eb) for m in mids)
    extra = {"config": {"n_seq": Ns, "lengths": f"uniform [{c['lo']}, {c['hi']}], seeded; "
                                                 f"mean {statistics.mean(lens):.0f}, total {sum(lens)} tokens",
                        "bits": c["bits"]}}
    print(json.dumps(_fixed_tier_line(args, ms, clocks, hot, layer_bytes, extra, 3 * L)), flush=True)


# --------------------------------------------------------------------------
# reassignment-time kernels (run on tier reassignment, not per decode step)
# --------------------------------------------------------------------------
def run_reassign(args):
    """Each reassignment kernel on inputs larger than L2, CUDA-event timed
    over --steps calls after --warmup: microseconds per call and achieved
    GB/s of its algorithmic bytes (every input read once, every output written
    once) against the measured HBM copy bandwidth.  Shapes: configuration 2's
    middle (16 x 8 x 8124 x 128, bf16) for the quantisers and the dequant;
    configuration 3's eviction (8 x 8 x 4096 -> 468 survivors, fp16; batch
    scaled x8 so the inputs exceed L2) for the re-RoPE gather."""
    import torch

    from fade_b200.quant import dequant_int4, quant_int2_grouped_packed, quant_k_int4, quant_v_int4
    from fade_b200.rope import Vanilla
    from fade_b200.rope_kernels import rerope_gather
    from fade_b200.rotated_quant import _random_orthogonal, rotated_quant_k, rotated_quant_v

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(9)
    B, H, S, D = 16, 8, 8124, 128
    x = torch.randn(B, H, S, D, device=dev, generator=gen).to(torch.bfloat16)
    n = x.numel()
    R = _random_orthogonal(D, 42).to(dev)
    kp, ks = quant_k_int4(x)
    vp, vs = quant_v_int4(x)
    S3, keep_n, B3 = 4096, 468, 64
    k3 = torch.randn(B3, 8, S3, D, device=dev, generator=gen).to(torch.float16)
    v3 = torch.randn_like(k3)
    keep = torch.sort(torch.randperm(S3, device=dev, generator=gen)[:keep_n]).values
    sc = Vanilla(theta=1e6, head_dim=D)
    co, so = sc.compute_cos_sin(torch.arange(S3, device=dev), dev, model_dtype=torch.float16)
    cn, sn = sc.compute_cos_sin(torch.arange(keep_n, device=dev), dev, model_dtype=torch.float16)
    co, so, cn, sn = (t.reshape(-1, D).contiguous() for t in (co, so, cn, sn))
    n3 = B3 * 8 * keep_n * D
    cases = [
        ("quant_int4_k (per-channel over S, pack)", lambda: quant_k_int4(x), n * 2 + n // 2 + B * H * D * 2),
        ("quant_int4_v (per-token, pack)", lambda: quant_v_int4(x), n * 2 + n // 2 + B * H * S * 2),
        ("quant_int2_grouped G=32 (4 codes per byte)", lambda: quant_int2_grouped_packed(x[:, :, :8096], 32),
         (n * 8096 // S) * 2 + (n * 8096 // S) // 4 + B * H * (8096 // 32) * D * 2),
        ("rotated_quant_k 2-bit (x R^T, per-channel)", lambda: rotated_quant_k(x, R, bits=2),
         n * 2 + n // 4 + B * H * D * 2),
        ("rotated_quant_v 2-bit (x R^T, per-token)", lambda: rotated_quant_v(x, R, bits=2),
         n * 2 + n // 4 + B * H * S * 2),
        ("dequant_int4 (K, per-channel scale)", lambda: dequant_int4(kp, ks, dtype=torch.bfloat16),
         n // 2 + B * H * D * 2 + n * 2),
        ("rerope_gather (un-RoPE + re-RoPE + gather K, gather V)",
         lambda: rerope_gather(k3, v3, keep, co, so, cn, sn), 4 * n3 * 2 + (S3 + keep_n) * D * 4 * 2),
    ]
    peaks = _measured_peaks()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    res = []
    for name, fn, nbytes in cases:
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / args.steps * 1e3
        gbs = nbytes / (us / 1e6) / 1e9
        res.append({"kernel": name, "us_per_call": round(us, 2), "algorithmic_bytes": int(nbytes),
                    "achieved_gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 3)})
    print(json.dumps({"reassignment_kernels": res, "peak_gbs": peak,
                      "note": "per call; each call allocates its outputs through torch (cached allocator)"}),
          flush=True)


def run_fade(args, ws, rank, local):
    kind = CFG["kind"]
    if kind == "int4":
        return run_int4(args, ws, rank, local)
    if ws > 1:
        raise SystemExit(f"config {CFG['id']} is a single-GPU workload")
    return (run_h2o if kind == "h2o" else run_rot)(args)


# --------------------------------------------------------------------------
# Hugging Face decode step through the reference's public API
# --------------------------------------------------------------------------
def run_hf(args):
    """One decode step of a random-init Llama-3.1-8B-shaped model (32 layers,
    hidden 4096, 32 q / 8 kv heads, head_dim 128, bf16; random weights: no
    checkpoints here) over config 2's batch and context, through
    create_tiered_cache + model.forward as a generate() loop runs it: the
    prompt is prefilled into the cache, each layer's middle is moved to INT4
    (4 sink + 64 recent tokens kept in bf16), then K decode steps (one token
    per sequence, greedy next token) are timed with CUDA events, once with the
    fused tiered attention and once with the cache materialised and passed to
    SDPA (fused_attention=False, the reference's decode path).  Host-side work
    of each step (HF's Python, the cache's bookkeeping) is inside the timing."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from fade_b200.cache import TIER_FP16, TIER_INT4
    from fade_b200.patch import create_tiered_cache

    c = CFG
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S = c["batch"], c["context"]
    L = c["layers"]
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=L,
                      num_attention_heads=c["n_q_heads"], num_key_value_heads=c["n_kv_heads"],
                      rope_theta=500000.0, max_position_embeddings=131072)
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).eval()
    torch.set_default_dtype(prev)
    gen = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (B, S - 1), device=dev, generator=gen)
    K, W = args.steps, max(3, args.warmup)
    res = {}
    from transformers import DynamicCache

    for mode in ("fused", "materialise", "dynamic"):
        if mode == "dynamic":   # transformers' own bf16 cache, no compression
            cache = DynamicCache()
        else:
            cache = create_tiered_cache(model, dtype=torch.bfloat16, n_sink=c["n_sink"],
                                        recent_window=c["recent"], fused_attention=(mode == "fused"))
        with torch.no_grad():
            nxt = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1).logits[:, -1]
            if mode != "dynamic":
                n = cache.get_seq_length(0)
                t = torch.full((n,), TIER_INT4, dtype=torch.long)
                t[:c["n_sink"]] = TIER_FP16
                t[n - c["recent"]:] = TIER_FP16
                for layer in range(L):
                    cache.apply_tier_assignment(layer, t)
            tok = nxt.argmax(-1, keepdim=True)
            for _ in range(W):
                tok = model(input_ids=tok, past_key_values=cache, use_cache=True,
                            logits_to_keep=1).logits[:, -1].argmax(-1, keepdim=True)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(K):
                tok = model(input_ids=tok, past_key_values=cache, use_cache=True,
                            logits_to_keep=1).logits[:, -1].argmax(-1, keepdim=True)
            e1.record()
            torch.cuda.synchronize(dev)
        res[mode] = e0.elapsed_time(e1) / K
        del cache
        torch.cuda.empty_cache()
    print(json.dumps({
        "metric": "HF decode step through create_tiered_cache (Llama-3.1-8B shape, random init)",
        "unit": "ms/step", "higher_is_better": False, "steps": K, "warmup": W, "dtype": "bf16",
        "data": "synthetic (random weights and prompt)",
        "config": {"workload": "config 2 shape as a whole model: 32 layers, batch 16, context 8192, "
                               "4 sink + 64 recent bf16, INT4 middle", "batch": B, "context": S, "layers": L},
        "fused_ms_per_step": round(res["fused"], 3), "materialise_sdpa_ms_per_step": round(res["materialise"], 3),
        "fused_tokens_per_s": round(B / (res["fused"] / 1e3), 1),
        "speedup": round(res["materialise"] / res["fused"], 2),
        "uncompressed_dynamic_cache_ms_per_step": round(res["dynamic"], 3),
    }), flush=True)


def main():
    args = parse()
    ws, rank, local = dist_env()
    if ws > 1:
        import torch.distributed as dist

        if args.impl == "fade":
            import torch

            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    try:
        if args.reassign:
            run_reassign(args)
        elif args.hf:
            run_hf(args)
        elif args.impl == "reference":
            run_reference(args, ws, rank)
        else:
            run_fade(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
