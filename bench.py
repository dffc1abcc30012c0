#!/usr/bin/env python
"""Benchmark of the cdl_b200 hot path; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload nvfp4_quant|mxfp4_quant|mxfp8_quant]

Default workload (``nvfp4_quant``): one step = NVFP4 quantize of one 4096x4096
bf16 activation tensor (N(0,1), seed 0, 0.1% x20
outliers; 16-element blocks, e4m3 scales, per-tensor alpha) through the
public ``nvfp4_quant`` API.  Inputs cycle through a pool of distinct tensors
totalling more than twice the 126 MB L2, so every step reads cold HBM.
Metric: algorithmic GB/s = 2.5625 B/element (2 B read, 0.5 B codes, 1/16 B
scales) x elements / time.

``value`` is timed with CUDA events over exactly K steps with the inputs
resident in HBM (max over ranks; each rank quantizes its own tensors, so
scaling is weak).  ``e2e`` is the same metric through the same API with the
input in pinned host memory: every step copies it host->device, quantizes,
and copies codes, scales and alpha back.

``--impl reference`` times the CPU implementation of the path (the oracle in
``oracle/``, a C restatement of cdl's torch quantize path, run on all host
threads) on rank 0 for the same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

WORKLOADS = {
    # name: (fmt, rows, k, bytes per element, config id)
    "nvfp4_quant": ("nvfp4", 4096, 4096, 2.5625, "C1"),
    "mxfp4_quant": ("mxfp4", 16384, 8192, 2.53125, "C2"),
    "mxfp8_quant": ("mxfp8", 16384, 8192, 3.03125, "C2"),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="nvfp4_quant")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--spinup-s", type=float, default=1.0, help="untimed clock ramp before warm-up")
    return ap.parse_args()


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def profile_traffic(workload: str) -> float | None:
    """DRAM bytes per step from the committed ncu summary of this workload."""
    p = os.path.join(ROOT, "profiles", f"{workload}.md")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_step:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU side: the oracle (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def cpu_quant_threads(x_bits, fmt_name: str, threads: int):
    """Oracle quantize of bf16 bits split by rows over `threads` host threads
    (ctypes releases the GIL).  NVFP4 computes the global amax first, as cdl."""
    import concurrent.futures

    import numpy as np

    import oracle

    fmt = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}[fmt_name]
    gmax = None
    if fmt == oracle.NVFP4:
        chunks = np.array_split(x_bits, threads)
        with concurrent.futures.ThreadPoolExecutor(threads) as ex:
            gms = list(ex.map(lambda c: oracle.nvfp4_global(c)[0], chunks))
        gmax = max(gms)
    parts = np.array_split(np.arange(x_bits.shape[0]), threads)
    with concurrent.futures.ThreadPoolExecutor(threads) as ex:
        outs = list(ex.map(lambda idx: oracle.quant(x_bits[idx[0]: idx[-1] + 1], fmt, gmax), parts))
    return outs


def cpu_rate(fmt_name: str, rows: int, k: int, bpe: float, steps: int, warmup: int, threads: int,
             target_s: float | None = None):
    """(GB/s, sample description, seconds) of the oracle on a bounded sample."""
    import numpy as np
    import torch

    from cdl_b200 import workloads

    x = workloads.c1_nvfp4(rows, k) if fmt_name == "nvfp4" else workloads.c2_mx(rows, k)
    bits = x.view(torch.int16).numpy().view(np.uint16)
    for _ in range(warmup):
        cpu_quant_threads(bits, fmt_name, threads)
    t0 = time.perf_counter()
    n = 0
    while n < steps or (target_s is not None and time.perf_counter() - t0 < target_s):
        cpu_quant_threads(bits, fmt_name, threads)
        n += 1
        if target_s is not None and n >= steps and time.perf_counter() - t0 >= target_s:
            break
    dt = time.perf_counter() - t0
    gbs = bpe * rows * k * n / dt / 1e9
    return gbs, f"{n} x {fmt_name} quantize of [{rows},{k}] bf16 ({threads} threads)", dt


# ---------------------------------------------------------------------------
def main() -> None:
    args = parse_args()
    fmt_name, rows, k, bpe, cfg = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    threads = len(os.sched_getaffinity(0))

    if args.impl == "reference":
        if rank != 0:
            return
        gbs, sample, _ = cpu_rate(fmt_name, rows, k, bpe, max(args.steps // 20, 3), min(args.warmup, 1), threads)
        print(json.dumps({
            "impl": "reference", "metric": f"{args.workload.replace('_quant', '')} quant GB/s",
            "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16->e2m1/e4m3", "data": "synthetic",
            "config": {"workload": f"{args.workload} {cfg} [{rows},{k}] bf16"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    import torch
    import torch.distributed as dist

    from cdl_b200 import workloads
    from cdl_b200.core.kernel import quant

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    qfn = {"nvfp4": quant.nvfp4_quant, "mxfp4": quant.mxfp4_quant, "mxfp8": quant.mxfp8_quant}[fmt_name]
    in_bytes = rows * k * 2
    pool_n = max(2, -(-2 * L2_BYTES // in_bytes))
    gen = workloads.c1_nvfp4 if fmt_name == "nvfp4" else workloads.c2_mx
    pool = [gen(rows, k, seed=1000 * rank + i, device=str(dev)) for i in range(pool_n)]
    alg_bytes = bpe * rows * k

    def barrier():
        if world > 1:
            dist.barrier()

    # spin-up (clock ramp + sampler coverage), then W warm-up steps
    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                           if os.environ.get("CUDA_VISIBLE_DEVICES") else local).start()
    t_end = time.time() + args.spinup_s
    i = 0
    while time.time() < t_end:
        qfn(pool[i % pool_n])
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize()
    for i in range(args.warmup):
        qfn(pool[i % pool_n])
    torch.cuda.synchronize()

    # device-resident timed region: exactly K steps, captured in one CUDA graph
    # (the API is capture-safe: no host sync, no cudaMalloc inside)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(3):
            qfn(pool[i % pool_n])
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graph_outs = [qfn(pool[i % pool_n]) for i in range(args.steps)]
    graph.replay()  # one full untimed replay on top of the W eager warm-up steps
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    clocks = sampler.stop()
    del graph_outs
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = alg_bytes * args.steps * world / (ms_max / 1e3) / 1e9

    # end to end through the public API with host buffers
    host_in = pool[0].cpu().pin_memory()
    p0, s0, a0 = qfn(pool[0])
    host_p = torch.empty(p0.shape, dtype=p0.dtype, pin_memory=True)
    host_s = torch.empty(s0.shape, dtype=s0.dtype, pin_memory=True)
    host_a = torch.empty(1, dtype=torch.float32, pin_memory=True)
    h2d = host_in.numel() * host_in.element_size()
    d2h = p0.numel() * p0.element_size() + s0.numel() + (4 if a0 is not None else 0)
    e2e_steps = max(3, min(args.steps, 50))

    def e2e_step():
        xd = host_in.to(dev, non_blocking=True)
        p, s, a = qfn(xd)
        host_p.copy_(p, non_blocking=True)
        host_s.copy_(s, non_blocking=True)
        if a is not None:
            host_a.copy_(a, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = alg_bytes * e2e_steps * world / (float(e2e_ms.item()) / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, sample, _ = cpu_rate(fmt_name, rows, k, bpe, 3, 1, threads, target_s=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}

    peaks, peak_src = load_peaks()
    per_step_s = ms_max / 1e3 / args.steps
    achieved = alg_bytes / per_step_s / 1e9
    traffic = profile_traffic(args.workload)
    launches_per_step = 1
    if rank == 0:
        print(json.dumps({
            "metric": f"{fmt_name.upper()} quant GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16->e2m1/e4m3" if fmt_name != "mxfp8" else "bf16->e4m3/e8m0",
            "data": "synthetic",
            "config": {"workload": f"{args.workload} {cfg} [{rows},{k}] bf16 per rank",
                       "l2": f"inputs cycled over {pool_n} tensors ({pool_n * in_bytes >> 20} MiB > 2x L2)",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "traffic": traffic, "peak_source": peak_src,
                         "kernel": "nvfp4_fused_kernel" if fmt_name == "nvfp4" else "quant_flat_kernel"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
