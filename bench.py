"""Benchmark: FADE tiered decode attention on B200.

Workload per GPU (weak scaling: every rank holds its own batch shard):
  Llama-3.1-8B-shaped decode, 32 layers, batch 16, 32 query / 8 KV heads,
  head_dim 128, bf16; context 8192 = 4 FP sink + 64 FP recent (ring) + 8124
  INT4 middle (K per-channel, V per-token, bit-packed).  One step = for every
  layer: age the oldest recent token into the INT4 middle (quantise + pack)
  and run the fused tiered decode attention of that layer's query.
  Synthetic N(0,1) K/V with 4 outlier channels per head x8, seeded.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fade|reference]
For N > 1 launch with torchrun (one process per GPU); the reported value is
the whole job's throughput and the step time is the max over ranks.
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

CFG = dict(layers=32, batch=16, n_q_heads=32, n_kv_heads=8, head_dim=128, context=8192, n_sink=4,
           recent=64, dtype="bf16")
METRIC = "tiered decode-attn effective KV GB/s (Llama-3.1-8B shape, 32 layers, step incl. age-out)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("fade", "reference"), default="fade")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--dtype", choices=("bf16", "f16"), default="bf16",
                    help="model dtype (the benchmark configuration is bf16)")
    ap.add_argument("--layers", type=int, default=CFG["layers"],
                    help="layers per step (profiling captures use 1; the benchmark is 32)")
    args = ap.parse_args()
    CFG["layers"] = args.layers
    CFG["dtype"] = args.dtype
    return args


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def algorithmic_bytes(n_mid: int, eb: int = 2, cfg=CFG, layers=None) -> tuple[int, int]:
    """(decode-attention bytes of one layer, age-out bytes of one layer) for one GPU's batch.
    Per (b, kv-head): FP tiers K+V, INT4 K and V codes (D/2 B each per token),
    per-token V scale, per-channel K scale, q read + out written for its g heads."""
    D, g = cfg["head_dim"], cfg["n_q_heads"] // cfg["n_kv_heads"]
    Z = cfg["batch"] * cfg["n_kv_heads"]
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
# reference arm (CPU): the reference's per-step path restated in oracle/
# --------------------------------------------------------------------------
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def time_cpu_reference(steps: int, warmup: int, threads: int):
    """Seconds per full 32-layer step, from single-layer samples x 32."""
    import torch

    from oracle.cpu_path import time_layer_steps

    n_mid = CFG["context"] - CFG["n_sink"] - CFG["recent"]
    dt = torch.bfloat16
    per_layer = time_layer_steps(CFG["batch"], CFG["n_q_heads"], CFG["n_kv_heads"], CFG["head_dim"],
                                 CFG["n_sink"], n_mid, CFG["recent"], dt, steps, warmup, threads)
    return [t * CFG["layers"] for t in per_layer], n_mid


def run_reference(args, ws, rank):
    if rank != 0:
        return
    threads = cpu_threads()
    steps = max(1, args.steps)
    step_s, n_mid = time_cpu_reference(steps, max(1, min(args.warmup, 3)), threads)
    dec_b, _ = algorithmic_bytes(n_mid)
    bytes_step = dec_b * CFG["layers"]
    t = statistics.mean(step_s)
    val = bytes_step / t / 1e9
    sample = (f"1 of {CFG['layers']} layers timed per step (x{CFG['layers']}): torch CPU cat(sink, cached "
              f"dequant middle, recent) + SDPA(enable_gqa) per the reference's decode path, batch "
              f"{CFG['batch']}, context {CFG['context']}")
    line = {
        "impl": "reference",
        "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_block(args.gpus),
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(n):
    return {"workload": "config 2: Llama-3.1-8B-shaped tiered decode (4 sink + 64 recent FP, 8124 INT4 middle)",
            "layers": CFG["layers"], "batch_per_gpu": CFG["batch"], "global_batch": CFG["batch"] * n,
            "n_q_heads": CFG["n_q_heads"], "n_kv_heads": CFG["n_kv_heads"], "head_dim": CFG["head_dim"],
            "context": CFG["context"], "parallelism": f"batch-sharded x{n} (weak)",
            "l2": "inputs larger than L2 (4.5 GB of compressed KV per step vs 126 MB L2)"}


# --------------------------------------------------------------------------
# fade arm (GPU)
# --------------------------------------------------------------------------
def _torch_dtype():
    import torch

    return {"bf16": torch.bfloat16, "f16": torch.float16}[CFG["dtype"]]


def build_decoder(dev, total_steps, shard_start: int = 0):
    import torch

    from fade_b200.decoder import TieredDecoder

    n_mid = CFG["context"] - CFG["n_sink"] - CFG["recent"]
    dec = TieredDecoder(CFG["layers"], CFG["batch"], CFG["n_q_heads"], CFG["n_kv_heads"], CFG["head_dim"],
                        dtype=_torch_dtype(), n_sink=CFG["n_sink"], recent_window=CFG["recent"],
                        mid_capacity=n_mid + total_steps + 8, device=dev)
    gen = torch.Generator(device=dev)
    B, H, S, D = CFG["batch"], CFG["n_kv_heads"], CFG["context"], CFG["head_dim"]
    for layer in range(CFG["layers"]):
        gen.manual_seed(1000 + layer + 100003 * shard_start)   # this rank's rows of the global batch
        k = torch.randn(B, H, S, D, device=dev, generator=gen)
        v = torch.randn(B, H, S, D, device=dev, generator=gen)
        for h in range(H):
            ch = torch.randperm(D, device=dev, generator=gen)[:4]
            k[:, h, :, ch] *= 8.0
            v[:, h, :, ch] *= 8.0
        dec.load_prompt(layer, k.to(_torch_dtype()), v.to(_torch_dtype()))
        del k, v
    torch.cuda.synchronize(dev)
    return dec, n_mid


def run_fade(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from fade_b200.shard import batch_shard, gather_objects, max_over_ranks

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    K, W = args.steps, max(3, args.warmup)
    roof_steps = min(K, 10)
    e2e_steps = 0 if args.no_e2e else min(K, 20)
    total = 2 + W + K + roof_steps + e2e_steps
    start, rows = batch_shard(CFG["batch"] * ws, ws, rank)   # weak scaling: CFG["batch"] rows per GPU
    assert rows == CFG["batch"]
    dec, n_mid0 = build_decoder(dev, total, start)
    L = CFG["layers"]
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    q = torch.randn(dec.q.shape, device=dev, generator=gen).to(_torch_dtype())
    kn = torch.randn(dec.k_new.shape, device=dev, generator=gen).to(_torch_dtype())
    vn = torch.randn(dec.v_new.shape, device=dev, generator=gen).to(_torch_dtype())
    dec.step(q, kn, vn)                      # eager step: builds plans, validates
    torch.cuda.synchronize(dev)
    dec.capture()
    for _ in range(W):
        dec.replay()
    torch.cuda.synchronize(dev)
    dec.check_device_errors()
    n_mid_start = n_mid0 + 1 + W

    props = torch.cuda.get_device_properties(dev)
    bus = getattr(props, "pci_bus_id", None)
    bus_ids = [b for b in gather_objects(bus) if b is not None]
    sampler = ClockSampler(bus_ids) if rank == 0 else None

    # ---------------- timed region: K graph replays ----------------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.start()
        time.sleep(0.3)
    e0.record()
    for _ in range(K):
        dec.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_max = max_over_ranks(e0.elapsed_time(e1), dev)   # the job's step time: slowest rank
    dec.check_device_errors()

    # bytes over the timed steps (the middle grows by one token per step)
    tot_bytes = 0
    for i in range(K):
        d_b, a_b = algorithmic_bytes(n_mid_start + i + 1)
        tot_bytes += (d_b + a_b) * L
    step_ms = ms_max / K
    value = tot_bytes * ws / (ms_max / 1e3) / 1e9

    # ---------------- roofline ----------------
    # The step is nothing but the L per-layer calls of fade_decode_attn_age_out
    # (middle_kernel + finish_kernel, chained with programmatic dependent
    # launch so a layer's middle starts streaming while the previous layer's
    # finisher drains).  The average call duration is the timed region / (K*L).
    avg_ms = step_ms / L
    attn_bytes = tot_bytes / (K * L)
    achieved = attn_bytes / (avg_ms / 1e3) / 1e9
    # For reference: one call timed alone between CUDA events (this serialises
    # the layers, so it includes each call's full start-up and drain).
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(L)]
    g2 = dec.capture(layer_events=evs)
    durs = []
    for i in range(roof_steps):
        g2.replay()
        torch.cuda.synchronize(dev)
        durs.extend(a.elapsed_time(b) for a, b in evs)
    iso_us = statistics.mean(durs) * 1e3
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    try:
        tr = json.loads((ROOT / "profiles" / "decode_attn_traffic.json").read_text())
        traffic = tr.get("bytes_per_launch_scaled")
    except Exception:
        pass

    # ---------------- e2e through the public API with host buffers ----------------
    e2e = None
    if e2e_steps:
        qh = q.cpu().pin_memory()
        kh = kn.cpu().pin_memory()
        vh = vn.cpu().pin_memory()
        oh = torch.empty(dec.out.shape, dtype=dec.out.dtype).pin_memory()
        dec.step_host(qh, kh, vh, oh)
        dec.capture_host(qh, kh, vh, oh)   # copies overlap the layers, one graph per step
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
        n_e = n_mid_start + K + roof_steps + 1
        eb = sum((sum(algorithmic_bytes(n_e + i + 1)) * L) for i in range(e2e_steps))
        e2e = {"value": round(eb * ws / (e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": int(qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2),
               "d2h_bytes_per_step": int(oh.numel() * 2),
               "ms_per_step": round(e_ms / e2e_steps, 4)}

    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline and ws == 1:
        threads = cpu_threads()
        samples, _ = time_cpu_reference(3, 1, threads)
        t = statistics.mean(samples)
        dec_b, _ = algorithmic_bytes(n_mid0)
        cpu = {"value": round(dec_b * L / t / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": "3 single-layer steps x32 layers of the reference's per-step CPU path "
                         "(cat of cached dequant tiers + SDPA, torch CPU), batch 16, context 8192"}
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": round(step_ms, 4), "us_per_step": round(step_ms * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"int4 codes -> {CFG['dtype']} ({CFG['dtype']} MMA, f32 accumulate)", "data": "synthetic", "config": config_block(ws),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "fade_decode_attn_age_out per layer (middle_kernel + finish_kernel)",
                     "avg_launch_us": round(avg_ms * 1e3, 2), "bytes_per_launch": int(attn_bytes),
                     "isolated_call_us": round(iso_us, 2),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in peaks else "fallback"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 2 * L * K,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


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
        if args.impl == "reference":
            run_reference(args, ws, rank)
        else:
            run_fade(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
