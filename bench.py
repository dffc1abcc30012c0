#!/usr/bin/env python
"""Benchmark of the cdl_b200 hot path; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload NAME]

Workloads (synthetic data everywhere):

* ``qat_1.7b`` (default) -- config C5: one SmolLM2-1.7B NVFP4 QAT training
  step (forward, backward, clip + AdamW) on 4x2048 uniform random tokens per
  rank, backend ``nvfp4_qbwd`` (NVFP4 forward, dgrad and wgrad GEMMs); one
  CUDA graph per step, for N > 1 data parallel with the NCCL bf16 gradient
  all-reduces (issued from the backward hooks) captured in the same graph,
  ``--comm-sms`` (16) SMs left to NCCL during the backward pass.
  Metric: tokens/s over all ranks.  At N=1 the line
  also carries ``components``: the other BASELINE metrics (NVFP4 quantize
  GB/s on C1 and on a larger-than-L2 tensor, MXFP4 / MXFP8 on C2, the
  transposed requantizes, the optimizer's weight encode, NVFP4 dequantize,
  FP4 GEMM TFLOP/s on C3 8192^3), each with its roofline, and, where they
  exist, the same workload through the reference's own Triton kernels
  (``reference_gpu``, from the unmodified reference package in
  ``baseline/_ref``) and through cuBLAS (``library_gpu``, the GEMM).
* ``qat_135m`` -- config C4 (8x2048 tokens).
* ``nvfp4_quant`` (C1 4096x4096), ``nvfp4_quant_large`` / ``nvfp4_quant_t``
  (C2 shape, row-wise / transposed), ``mxfp4_quant`` / ``mxfp8_quant`` (+
  ``_t``: C2 [16384, 8192]), ``nvfp4_dequant`` (C1), ``nvfp4_encode_multi``
  (the 1.7B model's 168 weights in one launch): one step = one call of the
  public API; inputs cycle through a pool larger than twice the 126 MB L2.
  Metric: algorithmic GB/s (2.5625 B/element for NVFP4).
* ``fp4_gemm`` -- config C3 (``--gemm-shape``, default 8192^3): one step =
  quantize the bf16 activations + the tcgen05 block-scaled GEMM against
  pre-quantized NVFP4 weights.  Metric: TFLOP/s (2 M N K per step).
* ``nvfp4_ecdl`` / ``nvfp4_ccdl`` -- the stochastic quantizers on C1.

Every step sequence is timed with CUDA events over exactly K steps with the
inputs resident in HBM (max over ranks; each rank processes its own data, so
scaling is weak).  ``e2e`` is the same metric through the same public API
with host-resident inputs: each step copies its input host->device and its
result back.  ``--impl reference`` times the reference's algorithm on the
host cores (rank 0): the CPU oracle (``oracle/``, a C restatement of cdl's
torch path) for the kernels, and for the QAT step the reference's training
step with its native-backend numerics (``oracle/qat_cpu.py``).
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
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
QUANT = {
    # name: (fmt, rows, k, bytes per element, config id[, transpose])
    "nvfp4_quant": ("nvfp4", 4096, 4096, 2.5625, "C1"),
    "mxfp4_quant": ("mxfp4", 16384, 8192, 2.53125, "C2"),
    "mxfp8_quant": ("mxfp8", 16384, 8192, 3.03125, "C2"),
    # the transposed (dim-0) requantize of the wgrad operands, C2 shape
    "mxfp4_quant_t": ("mxfp4", 16384, 8192, 2.53125, "C2 transposed", True),
    "mxfp8_quant_t": ("mxfp8", 16384, 8192, 3.03125, "C2 transposed", True),
    "nvfp4_quant_t": ("nvfp4", 16384, 8192, 2.5625, "C2 shape, transposed", True),
    # NVFP4 on a tensor twice the size of L2 (C1's 32 MiB fits in L2)
    "nvfp4_quant_large": ("nvfp4", 16384, 8192, 2.5625, "C2 shape"),
}
WORKLOADS = sorted(list(QUANT) + ["fp4_gemm", "qat_135m", "qat_1.7b", "nvfp4_ecdl", "nvfp4_ccdl",
                                  "nvfp4_encode_multi", "nvfp4_dequant", "nvfp4_dual"])
QAT_BATCH = {"qat_135m": (8, 2048), "qat_1.7b": (4, 2048)}  # configs C4 / C5, tokens per rank
ECDL_TOPK, ECDL_KAPPA = 5, 4.0  # theta_topk default of cdl's training config (smollm2.py:168)
CCDL_TOPK, CCDL_KAPPA = 5, 2.0  # cdl's training defaults (theta_topk = q_topk = 5, kappa 2)
CCDL_BPE = 2.0 + 4.0 / 16 + 0.5 + 1.0 / 16  # x, q (fp32 per block), codes, scale bytes


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=WORKLOADS, default="qat_1.7b")
    ap.add_argument("--no-components", action="store_true",
                    help="skip the N=1 component measurements (quantize GB/s, GEMM TFLOP/s)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--torch-profile", default="", metavar="PATH",
                    help="after the timed region, profile 2 more steps (CUDA kernels) and write the table to PATH")
    ap.add_argument("--backend", default="nvfp4_qbwd", choices=["nvfp4_qbwd", "nvfp4", "mxfp4", "mxfp8"],
                    help="QAT workloads: QLinear backend (nvfp4_qbwd = NVFP4 forward, dgrad and wgrad, the "
                         "configuration BASELINE names; nvfp4 = cdl's numerics: bf16 dgrad / wgrad)")
    ap.add_argument("--spinup-s", type=float, default=1.0, help="untimed clock ramp before warm-up")
    ap.add_argument("--no-graph", action="store_true", help="QAT workloads: eager steps even at N=1")
    ap.add_argument("--comm-sms", type=int, default=16,
                    help="QAT workloads, N > 1: SMs the backward pass's persistent kernels leave to NCCL "
                         "(also NCCL_MAX_CTAS unless set)")
    ap.add_argument("--gemm-shape", default="8192,8192,8192", metavar="M,N,K",
                    help="fp4_gemm: the GEMM shape (C3 is 8192^3; its sweep: M in {2048, 16384} x "
                         "(N, K) in {(2048, 8192), (8192, 2048), (49152, 576)})")
    a = ap.parse_args()
    qat = a.workload.startswith("qat")
    if a.steps is None:
        a.steps = 10 if qat else (20 if a.workload == "fp4_gemm" else 200)
    if a.warmup is None:
        a.warmup = 3 if qat else 10
    return a


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
        rows = [[p.strip() for p in line.split(",")] for line in open(self.path)]
        rows = [r for r in rows if len(r) >= 9]
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
            gmax = max(ex.map(lambda c: oracle.nvfp4_global(c)[0], chunks))
    parts = np.array_split(np.arange(x_bits.shape[0]), threads)
    with concurrent.futures.ThreadPoolExecutor(threads) as ex:
        return list(ex.map(lambda idx: oracle.quant(x_bits[idx[0]: idx[-1] + 1], fmt, gmax), parts))


def cpu_quant_rate(fmt_name, rows, k, bpe, steps, warmup, threads, target_s=None):
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
    dt = time.perf_counter() - t0
    return bpe * rows * k * n / dt / 1e9, f"{n} x {fmt_name} quantize of [{rows},{k}] bf16 ({threads} threads)"


def cpu_dual_rate(threads, target_s=10.0, rows=4096, k=4096):
    """The oracle's two NVFP4 quantizes the dual encoder replaces, of a bounded
    [rows, k] sample and of its transpose, in dual-encode GB/s (3.125 B per
    element)."""
    import numpy as np
    import torch

    from cdl_b200 import workloads

    bits = workloads.c2_mx(rows, k).view(torch.int16).numpy().view(np.uint16)
    bits_t = np.ascontiguousarray(bits.T)
    cpu_quant_threads(bits, "nvfp4", threads)
    t0 = time.perf_counter()
    n = 0
    while n < 2 or time.perf_counter() - t0 < target_s:
        cpu_quant_threads(bits, "nvfp4", threads)
        cpu_quant_threads(bits_t, "nvfp4", threads)
        n += 1
    dt = time.perf_counter() - t0
    return 3.125 * rows * k * n / dt / 1e9, (f"{n} x (nvfp4 quantize of [{rows},{k}] bf16 and of its transpose) "
                                             f"({threads} threads)")


def cpu_dequant_rate(threads, target_s=10.0, rows=4096, k=4096):
    """The oracle's NVFP4 dequantize of C1's encoding, rows split over
    ``threads`` host threads."""
    import concurrent.futures

    import numpy as np
    import torch

    import oracle
    from cdl_b200 import workloads

    bits = workloads.c1_nvfp4(rows, k).view(torch.int16).numpy().view(np.uint16)
    packed, scale, alpha = oracle.quant(bits, oracle.NVFP4)
    parts = np.array_split(np.arange(rows), threads)

    def run():
        with concurrent.futures.ThreadPoolExecutor(threads) as ex:
            list(ex.map(lambda idx: oracle.dequant(packed[idx[0]: idx[-1] + 1], scale[idx[0]: idx[-1] + 1],
                                                   oracle.NVFP4, alpha), parts))

    run()
    t0 = time.perf_counter()
    n = 0
    while n < 3 or time.perf_counter() - t0 < target_s:
        run()
        n += 1
    dt = time.perf_counter() - t0
    return 2.5625 * rows * k * n / dt / 1e9, f"{n} x nvfp4 dequantize of [{rows},{k}] ({threads} threads)"


def cpu_ecdl_rate(rows, k, threads, target_s=10.0):
    """The ECDL oracle (numpy restatement) on a bounded row sample of C1."""
    import numpy as np

    from cdl_b200 import workloads
    from oracle import ecdl as E

    x = workloads.c1_nvfp4(rows, k, seed=0).float().numpy().reshape(rows, k // 16, 16)
    sample_rows = 64
    t0, cnt = time.perf_counter(), 0
    while cnt < 1 or time.perf_counter() - t0 < target_s:
        E.forward(E.NVFP4, x[:sample_rows], ECDL_KAPPA, cnt + 1, ECDL_TOPK, E.MODE_NVIDIA)
        cnt += 1
    dt = time.perf_counter() - t0
    return (2.5625 * sample_rows * k * cnt / dt / 1e9,
            f"{cnt} x NVFP4 ECDL forward (numpy oracle) of {sample_rows}x{k} of C1 (1 thread)")


def _ccdl_q(x):
    """Per-block learnable scales as a CCDL weight quantizer initialises them:
    block amax / 6 (fp32), alpha 1."""
    return (x.float().abs().amax(-1) / 6.0).clamp_min(2.0 ** -126)


def cpu_ccdl_rate(rows, k, threads, target_s=10.0):
    """The CCDL oracle (numpy restatement) on a bounded row sample of C1."""
    import numpy as np

    from cdl_b200 import workloads
    from oracle import ecdl as E

    x = workloads.c1_nvfp4(rows, k, seed=0).reshape(rows, k // 16, 16)
    q = _ccdl_q(x).numpy()
    x = x.float().numpy()
    sample_rows = 64
    t0, cnt = time.perf_counter(), 0
    while cnt < 1 or time.perf_counter() - t0 < target_s:
        E.ccdl_forward(E.NVFP4, x[:sample_rows], q[:sample_rows], CCDL_KAPPA, CCDL_KAPPA, 1.0, cnt + 1, CCDL_TOPK,
                       CCDL_TOPK)
        cnt += 1
    dt = time.perf_counter() - t0
    return (CCDL_BPE * sample_rows * k * cnt / dt / 1e9,
            f"{cnt} x NVFP4 CCDL forward (numpy oracle) of {sample_rows}x{k} of C1 (1 thread)")


def ccdl_workload(dev, rank):
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel.ccdl import ccdl_quant_fwd
    from cdl_b200.core.kernel.ecdl import FormatId

    rows, k = QUANT["nvfp4_quant"][1:3]
    pool_n = max(2, -(-2 * L2_BYTES // (rows * k * 2)))
    pool = [workloads.c1_nvfp4(rows, k, seed=1000 * rank + i, device=str(dev)).reshape(rows, k // 16, 16)
            for i in range(pool_n)]
    qs = [_ccdl_q(x) for x in pool]
    kt = torch.tensor(CCDL_KAPPA, device=dev)
    kq = torch.tensor(CCDL_KAPPA, device=dev)
    alpha = torch.ones((), device=dev)
    seeds = [torch.tensor(i + 1, dtype=torch.int64, device=dev) for i in range(pool_n)]
    host_in, host_q = pool[0].cpu().pin_memory(), qs[0].cpu().pin_memory()

    def run(x, q, seed):
        return ccdl_quant_fwd(x, q, kt, kq, alpha, seed, int(FormatId.NVFP4), CCDL_TOPK, CCDL_TOPK)

    p0, s0 = run(pool[0], qs[0], seeds[0])
    host_p = torch.empty(p0.shape, dtype=p0.dtype, pin_memory=True)
    host_s = torch.empty(s0.shape, dtype=s0.dtype, pin_memory=True)

    def e2e_step():
        p, s_ = run(host_in.to(dev, non_blocking=True), host_q.to(dev, non_blocking=True), seeds[0])
        host_p.copy_(p, non_blocking=True)
        host_s.copy_(s_, non_blocking=True)

    return {
        "step": lambda i: run(pool[i % pool_n], qs[i % pool_n], seeds[i % pool_n]),
        "e2e_step": e2e_step, "graph": True,
        "units_per_step": CCDL_BPE * rows * k / 1e9, "unit": "GB/s", "metric": "NVFP4 CCDL quant GB/s",
        "dtype": "bf16->e2m1 with sampled ue4m3 scales (stochastic, Philox)",
        "config": {"workload": f"nvfp4_ccdl C1 [{rows},{k}] bf16 per rank, theta_topk {CCDL_TOPK}, q_topk "
                               f"{CCDL_TOPK}, kappa {CCDL_KAPPA}, q from block amax",
                   "l2": f"inputs cycled over {pool_n} tensors (> 2x L2)"},
        "h2d": host_in.numel() * 2 + host_q.numel() * 4, "d2h": p0.numel() + s0.numel(),
        "bound": "hbm", "kernel": "ccdl_fwd_kernel",
        "launches_per_step": 1,
    }


def ecdl_workload(dev, rank):
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel.ecdl import FormatId, ecdl_quant_fwd

    rows, k = QUANT["nvfp4_quant"][1:3]
    pool_n = max(2, -(-2 * L2_BYTES // (rows * k * 2)))
    pool = [workloads.c1_nvfp4(rows, k, seed=1000 * rank + i, device=str(dev)).reshape(rows, k // 16, 16)
            for i in range(pool_n)]
    kappa = torch.tensor(ECDL_KAPPA, device=dev)
    seeds = [torch.tensor(i + 1, dtype=torch.int64, device=dev) for i in range(pool_n)]
    host_in = pool[0].cpu().pin_memory()
    p0, s0, _ = ecdl_quant_fwd(pool[0], kappa, seeds[0], FormatId.NVFP4, ECDL_TOPK, "nvidia")
    host_p = torch.empty(p0.shape, dtype=p0.dtype, pin_memory=True)
    host_s = torch.empty(s0.shape, dtype=s0.dtype, pin_memory=True)

    def e2e_step():
        p, s_, _ = ecdl_quant_fwd(host_in.to(dev, non_blocking=True), kappa, seeds[0], FormatId.NVFP4, ECDL_TOPK,
                                  "nvidia")
        host_p.copy_(p, non_blocking=True)
        host_s.copy_(s_, non_blocking=True)

    return {
        "step": lambda i: ecdl_quant_fwd(pool[i % pool_n], kappa, seeds[i % pool_n], FormatId.NVFP4, ECDL_TOPK,
                                         "nvidia"),
        "e2e_step": e2e_step, "graph": True,
        "units_per_step": 2.5625 * rows * k / 1e9, "unit": "GB/s", "metric": "NVFP4 ECDL quant GB/s",
        "dtype": "bf16->e2m1/e4m3 (stochastic, Philox)",
        "config": {"workload": f"nvfp4_ecdl C1 [{rows},{k}] bf16 per rank, theta_topk {ECDL_TOPK}, "
                               f"kappa {ECDL_KAPPA}, nvidia scales",
                   "l2": f"inputs cycled over {pool_n} tensors (> 2x L2)"},
        "h2d": host_in.numel() * 2, "d2h": p0.numel() + s0.numel(),
        "bound": "hbm", "kernel": "ecdl_fwd_kernel (+ ecdl_amax_kernel)",
        "launches_per_step": 2,
    }


def cpu_gemm_rate(threads, target_s=10.0):
    """Oracle NVFP4 GEMM (quantize A, dequantize, fp32 matmul) on a 2048^3 sample."""
    import numpy as np
    import torch

    import oracle
    from cdl_b200 import workloads

    torch.set_num_threads(threads)
    m = n = k = 2048
    a, w = workloads.c3_gemm(m, n, k)
    ab = a.view(torch.int16).numpy().view(np.uint16)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    wp, ws, wa = oracle.quant(wb, oracle.NVFP4)
    t0, cnt = time.perf_counter(), 0
    while cnt < 1 or time.perf_counter() - t0 < target_s:
        ap, as_, aa = oracle.quant(ab, oracle.NVFP4)
        oracle.mm(ap, as_, wp, ws, oracle.NVFP4, float(aa[0] * wa[0]))
        cnt += 1
    dt = time.perf_counter() - t0
    return (2.0 * m * n * k * cnt / dt / 1e12,
            f"{cnt} x NVFP4 quantize(A) + dequantize + fp32 matmul at {m}^3 ({threads} threads)")


def cpu_qat_rate(workload, threads):
    """The CPU NVFP4 QAT step with the reference's native-backend numerics
    (``oracle/qat_cpu.py``): one step of the full model on a 1x256-token
    sample, its fixed per-step weight quantize timed apart, projected to the
    workload's tokens per step."""
    from cdl_b200.train import qat
    from oracle import qat_cpu

    spec = qat.SPECS["135m" if workload == "qat_135m" else "1.7b"]
    batch, seq = QAT_BATCH[workload]
    return qat_cpu.qat_step_rate(spec, 1, 256, threads, steps=1, full_tokens=batch * seq)


# ---------------------------------------------------------------------------
# GPU workloads
# ---------------------------------------------------------------------------
def quant_workload(name, dev, rank):
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel import quant

    fmt, rows, k, bpe, cfg = QUANT[name][:5]
    tr = len(QUANT[name]) > 5 and QUANT[name][5]
    qf = {"nvfp4": quant.nvfp4_quant, "mxfp4": quant.mxfp4_quant, "mxfp8": quant.mxfp8_quant}[fmt]

    def qfn(x):
        return qf(x, transpose=tr)

    in_bytes = rows * k * 2
    pool_n = max(2, -(-2 * L2_BYTES // in_bytes))
    gen = workloads.c1_nvfp4 if fmt == "nvfp4" else workloads.c2_mx
    pool = [gen(rows, k, seed=1000 * rank + i, device=str(dev)) for i in range(pool_n)]
    host_in = pool[0].cpu().pin_memory()
    p0, s0, a0 = qfn(pool[0])
    host_p = torch.empty(p0.shape, dtype=p0.dtype, pin_memory=True)
    host_s = torch.empty(s0.shape, dtype=s0.dtype, pin_memory=True)
    host_a = torch.empty(1, dtype=torch.float32, pin_memory=True)

    def e2e_step():
        p, s, a = qfn(host_in.to(dev, non_blocking=True))
        host_p.copy_(p, non_blocking=True)
        host_s.copy_(s, non_blocking=True)
        if a is not None:
            host_a.copy_(a, non_blocking=True)

    if tr:  # the C2 shapes take the tiled column kernels (rows % 64 == 0, k % 128 == 0)
        kernel, launches = (("nvfp4_dual_multi_kernel, column pass (+ amax_kernel)", 2) if fmt == "nvfp4"
                            else ("mx_col_kernel", 1))
    else:
        kernel, launches = ("nvfp4_fused_kernel" if fmt == "nvfp4" else "quant_flat_kernel"), 1
    w = {
        "step": lambda i: qfn(pool[i % pool_n]), "e2e_step": e2e_step, "graph": True,
        "units_per_step": bpe * rows * k / 1e9, "unit": "GB/s", "metric": f"{fmt.upper()} quant GB/s",
        "dtype": "bf16->e2m1/e4m3" if fmt != "mxfp8" else "bf16->e4m3/e8m0",
        "config": {"workload": f"{name} {cfg} [{rows},{k}] bf16 per rank" + (", blocks along dim 0" if tr else ""),
                   "l2": f"inputs cycled over {pool_n} tensors ({pool_n * in_bytes >> 20} MiB > 2x L2)"},
        "h2d": host_in.numel() * 2, "d2h": p0.numel() * p0.element_size() + s0.numel() + (4 if a0 is not None else 0),
        "bound": "hbm", "kernel": kernel, "launches_per_step": launches,
    }
    ref = reference_kernels()
    if ref is not None:
        rfn = getattr(ref[0], f"{fmt}_quant")
        # cdl has no transposed quantize: its caller quantizes a transposed copy
        w["reference_step"] = ((lambda i: rfn(pool[i % pool_n].t().contiguous())) if tr
                               else (lambda i: rfn(pool[i % pool_n])))
        w["reference_impl"] = (f"cdl.core.kernel.quant.{fmt}_quant (Triton _quant_kernel"
                               + (", torch amax" if fmt == "nvfp4" else "") + ")"
                               + (" of x.t().contiguous()" if tr else ""))
    return w


def reference_kernels():
    """cdl's own quantize / dequantize modules (Triton kernels), from the
    unmodified reference package installed under ``baseline/_ref``; None
    when it is not installed or does not import."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "cdl")):
        return None
    if ref not in sys.path:
        sys.path.append(ref)
    try:
        import cdl.core.kernel.dequant as rdq
        import cdl.core.kernel.quant as rq
    except Exception:
        return None
    return rq, rdq


def dequant_workload(dev, rank):
    """NVFP4 dequantize on C1 (4096 x 4096): codes + linear scales + alpha ->
    bf16, the operand cdl's bf16 backward reads (``dequant.py:103-109``)."""
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel import dequant, quant

    rows, k = 4096, 4096
    pool_n = 8
    pool = [quant.nvfp4_quant(workloads.c1_nvfp4(rows, k, seed=1000 * rank + i, device=str(dev)))
            for i in range(pool_n)]
    host = [t.cpu().pin_memory() for t in pool[0]]
    host_out = torch.empty(rows, k, dtype=torch.bfloat16, pin_memory=True)

    def e2e_step():
        p, s, a = (t.to(dev, non_blocking=True) for t in host)
        host_out.copy_(dequant.nvfp4_dequant(p, s, a), non_blocking=True)

    w = {
        "step": lambda i: dequant.nvfp4_dequant(*pool[i % pool_n]), "e2e_step": e2e_step, "graph": True,
        "units_per_step": 2.5625 * rows * k / 1e9, "unit": "GB/s", "metric": "NVFP4 dequant GB/s",
        "dtype": "e2m1/e4m3->bf16",
        "config": {"workload": f"nvfp4_dequant C1 [{rows},{k}] per rank",
                   "l2": f"inputs cycled over {pool_n} encodings, {pool_n} x 32 MiB of outputs (> 2x L2)"},
        "h2d": sum(t.numel() * t.element_size() for t in host), "d2h": rows * k * 2,
        "bound": "hbm", "kernel": "fp4_dequant32_kernel", "launches_per_step": 1,
    }
    ref = reference_kernels()
    if ref is not None:
        w["reference_step"] = lambda i: ref[1].nvfp4_dequant(*pool[i % pool_n])
        w["reference_impl"] = "cdl.core.kernel.dequant.nvfp4_dequant (Triton _fp4_dequant_kernel)"
    return w


def dual_workload(dev, rank, shape=(8192, 8192)):
    """The dual NVFP4 encode of the quantized backward (``nvfp4_dual_quant``):
    ``Q(x)`` and ``Q(x^T)`` of one bf16 [R, C] tensor from one read, amax
    given (as from a producer kernel's epilogue).  Default [8192, 8192]: the
    1.7B step's gate / up gradients (8192 tokens x 8192)."""
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel.quant import nvfp4_amax, nvfp4_dual_quant

    r, c = shape
    in_bytes = r * c * 2
    pool_n = max(2, -(-2 * L2_BYTES // in_bytes))
    pool = [workloads.c2_mx(r, c, seed=1000 * rank + i, device=str(dev)) for i in range(pool_n)]
    gmax = [nvfp4_amax(x)[0] for x in pool]
    host_in = pool[0].cpu().pin_memory()
    (p0, s0, _), (q0, t0, _) = nvfp4_dual_quant(pool[0], gmax=gmax[0])
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (p0, s0, q0, t0)]

    def e2e_step():
        x = host_in.to(dev, non_blocking=True)
        (p, s, _), (q, t, _) = nvfp4_dual_quant(x)
        for h, d in zip(host_out, (p, s, q, t)):
            h.copy_(d, non_blocking=True)

    return {
        "step": lambda i: nvfp4_dual_quant(pool[i % pool_n], gmax=gmax[i % pool_n]), "e2e_step": e2e_step,
        "graph": True, "units_per_step": 3.125 * r * c / 1e9, "unit": "GB/s",
        "metric": "NVFP4 dual encode GB/s", "dtype": "bf16->e2m1/e4m3 (rows and columns)",
        "config": {"workload": f"nvfp4_dual [{r},{c}] bf16 per rank: Q(x) and Q(x^T), amax given",
                   "l2": f"inputs cycled over {pool_n} tensors ({pool_n * in_bytes >> 20} MiB > 2x L2)"},
        "h2d": in_bytes, "d2h": sum(t.numel() for t in (p0, s0, q0, t0)),
        "bound": "hbm", "kernel": "nvfp4_dual_multi_kernel", "launches_per_step": 1,
    }


def encode_multi_workload(dev, rank, spec_name="1.7b", with_deq=True):
    """The QAT step's weight re-encode: one ``cdlb200_nvfp4_encode_multi``
    launch over the 168 quantized weights of SmolLM2-1.7B (N(0, 0.02)), amax
    given (the optimizer forms it), codes + GEMM-layout scales + alpha and,
    for the bf16 backward, the dequantized copy."""
    import ctypes

    import torch

    from cdl_b200 import _lib
    from cdl_b200.train import qat

    spec = qat.SPECS[spec_name]
    h, f = spec.hidden, spec.intermediate
    kvd = spec.kv_heads * (h // spec.heads)
    shapes = [(h, h), (kvd, h), (kvd, h), (h, h), (f, h), (f, h), (h, f)] * spec.layers
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    ws = [(torch.randn(r, c, generator=g, device=dev) * 0.02).to(torch.bfloat16) for r, c in shapes]
    amax = torch.stack([w.abs().max().float() for w in ws]).to(torch.bfloat16).view(torch.int16).to(torch.int32)
    amax = amax & 0x7FFF
    table = (_lib.Nvfp4EncodeTensor * len(ws))()
    bufs = []
    for j, w in enumerate(ws):
        r, c = w.shape
        b = (torch.empty(r, c // 2, dtype=torch.uint8, device=dev), torch.empty(r, c // 16, dtype=torch.uint8,
             device=dev), torch.empty(1, dtype=torch.float32, device=dev),
             torch.empty(r, c, dtype=torch.bfloat16, device=dev) if with_deq else None)
        bufs.append(b)
        t = table[j]
        t.x, t.rows, t.k, t.amax, t.amax_words = w.data_ptr(), r, c, amax.data_ptr() + 4 * j, 1
        t.packed, t.scale, t.alpha, t.deq = b[0].data_ptr(), b[1].data_ptr(), b[2].data_ptr(), _lib.ptr(b[3])
    n = sum(w.numel() for w in ws)
    bpe = 2 + 0.5 + 1 / 16 + (2 if with_deq else 0)

    def step(i=0):
        _lib.call("cdlb200_nvfp4_encode_multi", ctypes.addressof(table), len(ws), _lib.stream(dev))

    return {
        "step": step, "e2e_step": step, "graph": True, "keep": (ws, bufs, amax, table),
        "units_per_step": bpe * n / 1e9, "unit": "GB/s", "metric": "NVFP4 weight encode GB/s",
        "dtype": "bf16->e2m1/ue4m3 (+ bf16 dequantized copy)" if with_deq else "bf16->e2m1/ue4m3",
        "config": {"workload": f"nvfp4_encode_multi: the {len(ws)} quantized weights of {spec.name} "
                               f"({n / 1e9:.2f} G elements) in one launch, amax given",
                   "l2": f"{2 * n / 2**30:.1f} GiB of inputs >> L2"},
        "h2d": 0, "d2h": 0, "bound": "hbm", "kernel": "nvfp4_encode_multi_kernel", "launches_per_step": 1,
    }


def gemm_workload(dev, rank, shape=(8192, 8192, 8192)):
    import torch

    from cdl_b200 import workloads
    from cdl_b200.core.kernel import quant
    from cdl_b200.core.mm.swizzle import swizzle_scale_factors
    from cdl_b200.model.wrapper.ops import mm_nvfp4_alpha2

    m, n, k = shape
    pool_n = max(2, -(-2 * L2_BYTES // (m * k * 2)))  # bf16 A cycled over more than twice L2
    pool = []
    for i in range(pool_n):
        a, w = workloads.c3_gemm(m, n, k, seed=100 * rank + i, device=str(dev))
        pool.append(a)
    wp, wsf, wal = quant.nvfp4_quant(w)
    wsw = swizzle_scale_factors(wsf)

    def step(i):
        ap, asf, aal = quant.nvfp4_quant(pool[i % pool_n], swizzled=True)
        return mm_nvfp4_alpha2(ap, wp.T, asf, wsw.T, aal, wal)

    # the GEMM kernel alone (A already quantized), for the roofline of the dominant kernel
    pre = [quant.nvfp4_quant(a, swizzled=True) for a in pool]

    def kernel_step(i):
        ap, asf, aal = pre[i % pool_n]
        return mm_nvfp4_alpha2(ap, wp.T, asf, wsw.T, aal, wal)

    host_a = pool[0].cpu().pin_memory()
    host_out = torch.empty(m, n, dtype=torch.bfloat16, pin_memory=True)

    def e2e_step():
        ap, asf, aal = quant.nvfp4_quant(host_a.to(dev, non_blocking=True), swizzled=True)
        host_out.copy_(mm_nvfp4_alpha2(ap, wp.T, asf, wsw.T, aal, wal), non_blocking=True)

    def library_step(i):
        """The same GEMM through cuBLAS's NVFP4 path (torch scaled_mm), for comparison."""
        from torch.nn.functional import ScalingType, SwizzleType, scaled_mm

        ap, asf, aal = pre[i % pool_n]
        f4 = torch.float4_e2m1fn_x2
        return scaled_mm(ap.view(f4), wp.view(f4).T, [asf.view(torch.float8_e4m3fn).flatten(), aal],
                         [ScalingType.BlockWise1x16, ScalingType.TensorWise],
                         [wsw.view(torch.float8_e4m3fn).flatten(), wal],
                         [ScalingType.BlockWise1x16, ScalingType.TensorWise],
                         swizzle_a=[SwizzleType.SWIZZLE_32_4_4, SwizzleType.NO_SWIZZLE],
                         swizzle_b=[SwizzleType.SWIZZLE_32_4_4, SwizzleType.NO_SWIZZLE],
                         output_dtype=torch.bfloat16)

    return {
        "step": step, "e2e_step": e2e_step, "kernel_step": kernel_step, "graph": True,
        "library_step": library_step, "library_impl": "cuBLAS NVFP4 (torch.nn.functional.scaled_mm, 1x16 blocks)",
        "units_per_step": 2.0 * m * n * k / 1e12, "unit": "TFLOP/s", "metric": "FP4 GEMM TFLOPS",
        "dtype": "e2m1 x e2m1 (ue4m3 block scales) -> fp32 acc -> bf16",
        "config": {"workload": f"fp4_gemm C3 NVFP4 {m}x{n}x{k}: quantize bf16 A + tcgen05 GEMM vs pre-quantized W",
                   "l2": f"A cycled over {pool_n} tensors of {m * k * 2 / 2**20:.0f} MiB (> 2x L2 in total)"},
        "h2d": host_a.numel() * 2, "d2h": m * n * 2, "bound": "tensor",
        "kernel": "bs_gemm_pair_kernel<NVFP4> (persistent 2-SM tcgen05 block-scaled GEMM)",
        "launches_per_step": 2,  # nvfp4_fused_kernel (A), the GEMM (alpha_a * alpha_b in its epilogue)
    }


def qat_workload(name, dev, rank, world, backend="nvfp4", use_graph=True, comm_sms=16):
    import torch

    from cdl_b200.train import qat

    spec = qat.SPECS["135m" if name == "qat_135m" else "1.7b"]
    batch, seq = QAT_BATCH[name]
    # one process per GPU: the whole step is one CUDA graph, data parallel
    # too (the NCCL all-reduces issued from the backward hooks are captured)
    graph = use_graph
    step = qat.QatStep(spec, dev, backend=backend, seed=0, ddp=world > 1, graph=graph, comm_sms=comm_sms)
    qbwd = backend.endswith("_qbwd")
    pool = [qat.random_tokens(batch, seq, spec.vocab, seed=1000 * rank + i, device=dev) for i in range(4)]
    host_ids = pool[0].cpu().pin_memory()
    host_loss = torch.empty(1, dtype=torch.float32, pin_memory=True)

    def e2e_step():
        loss, _ = step.step(host_ids.to(dev, non_blocking=True))
        host_loss.copy_(loss.float().reshape(1), non_blocking=True)

    return {
        "step": lambda i: step.step(pool[i % len(pool)]), "e2e_step": e2e_step, "graph": False,
        "units_per_step": batch * seq, "unit": "tokens/s", "metric": "SmolLM2 NVFP4 QAT tokens/s",
        "dtype": ("nvfp4 fwd/dgrad/wgrad GEMMs (e2m1/ue4m3)" if qbwd else
                  "nvfp4 fwd GEMMs (e2m1/ue4m3), bf16 dgrad/wgrad as cdl") + ", bf16 params, clip + AdamW "
                 f"({step.optimizer})",
        "config": {"workload": f"{name} {'C4' if name == 'qat_135m' else 'C5'} {spec.name} QAT step, "
                               f"{batch}x{seq} tokens per rank, AdamW lr 3e-4, backend {backend}",
                   "backend": backend, "comm_sms": step.comm_sms,
                   "model": spec.name, "global_batch": batch * world, "seq_len": seq,
                   "parallelism": f"dp{world}" if world > 1 else "single", "l2": "activations >> L2"},
        "h2d": host_ids.numel() * 8, "d2h": 4, "bound": "tensor",
        "flops_per_unit": qat.flops_per_token(spec, seq),
        "kernel": "full QAT step (one CUDA graph per step)" if graph else "full QAT step (eager)",
        # eager steps: the library counts its kernel launches as they are
        # issued; a graph step replays the launches counted at its capture
        "launches_per_step": None, "count_launches": True,
        "graph_launches": (lambda: getattr(step, "graph_launches", 0)) if graph else None,
        "check_status": step.check_status,
        "release": step.release_graph,
    }


def time_steps(w, steps, dev):
    """Returns a callable running exactly `steps` steps (graph-captured when
    the workload allows it) and the captured outputs to keep alive."""
    import torch

    if not w["graph"]:
        def run():
            for i in range(steps):
                w["step"](i)

        return run, None
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(3):
            w["step"](i)
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = [w["step"](i) for i in range(steps)]
    g.replay()
    torch.cuda.synchronize()
    return g.replay, (g, outs)


FP4_PEAK_NOTE = ("denominator = 4 x the measured cuBLAS bf16 burst peak: the block-scaled FP4 MMA retires "
                 "4x the K of a bf16 MMA per cycle (measured on this pool: 128 cycles for M128 N256 K64 FP4 "
                 "and for K16 bf16); nominal dense FP4 is 9 PFLOP/s")


def time_kernel(fn, steps, dev):
    """Average device time (ms) of ``fn(i)`` over ``steps`` launches replayed
    from one CUDA graph (so that a short kernel is not timed at the host's
    launch rate)."""
    return graph_ms(fn, steps, 3, dev) / steps


def reference_qat_gpu(workload, dev, steps, warmup):
    """The reference's own QAT step (``baseline/reference_step.py``: cdl's
    QLinear + SteQuant("nvfp4") with its Triton quantizers, the native
    backend, Liger's loss, torch AdamW) on the same workload and GPU, eager as
    the reference's script runs it; None when the reference is not installed."""
    import torch

    from baseline import reference_step
    from cdl_b200.train import qat

    if reference_step.unavailable() is not None:
        return {"impl": "cdl smollm2.py step (native backend)", "unavailable": reference_step.unavailable()}
    spec = qat.SPECS["135m" if workload == "qat_135m" else "1.7b"]
    batch, seq = QAT_BATCH[workload]
    ref = reference_step.ReferenceQatStep(spec, dev, lr=3e-4, seed=0)
    gen = torch.Generator(device=dev).manual_seed(1)
    ids = [torch.randint(0, spec.vocab, (batch, seq), device=dev, generator=gen) for _ in range(2)]
    for i in range(warmup):
        ref.step(ids[i % 2])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        ref.step(ids[i % 2])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del ref
    return {"impl": "cdl smollm2.py step: QLinear + SteQuant('nvfp4') (Triton quantize / dequantize), native "
                    "backend (bf16 cuBLAS matmuls), Liger fused linear CE, torch AdamW; eager",
            "value": round(batch * seq / (ms / 1e3), 2), "unit": "tokens/s", "ms_per_step": round(ms, 3),
            "steps": steps}


def graph_ms(step, steps, warmup, dev):
    """Device time (ms) of ``steps`` calls of ``step(i)``, captured in one CUDA
    graph after ``warmup`` eager calls."""
    import torch

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    run, keep = time_steps({"graph": True, "step": step}, steps, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del keep, run
    return ms


def reference_gpu(w, steps, warmup, dev, key="reference"):
    """The reference's own GPU implementation of the workload (``key`` =
    "reference"), or a library's (``key`` = "library"), timed like this
    library's kernels (same inputs, one CUDA graph); None when there is none,
    ``{"unavailable": reason}`` when it raises."""
    if f"{key}_step" not in w:
        return None
    try:
        ms = graph_ms(w[f"{key}_step"], steps, warmup, dev)
    except Exception as e:  # a Python-level error of the other implementation, not of this library
        return {"impl": w[f"{key}_impl"], "unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
    return {"impl": w[f"{key}_impl"], "value": round(w["units_per_step"] * steps / (ms / 1e3), 2),
            "unit": w["unit"], "ms_per_step": round(ms / steps, 5)}


def measure_component(name, dev, steps, warmup, peaks):
    """Device-timed throughput and roofline of one kernel-level workload (N=1)."""
    if name in QUANT:
        w = quant_workload(name, dev, 0)
    elif name == "nvfp4_encode_multi":
        w = encode_multi_workload(dev, 0)
    elif name == "nvfp4_dequant":
        w = dequant_workload(dev, 0)
    elif name == "nvfp4_dual":
        w = dual_workload(dev, 0)
    else:
        w = gemm_workload(dev, 0)
    ms = graph_ms(w["step"], steps, warmup, dev)
    value = w["units_per_step"] * steps / (ms / 1e3)
    achieved = value
    if "kernel_step" in w:  # the dominant kernel alone
        achieved = w["units_per_step"] / (time_kernel(w["kernel_step"], steps, dev) / 1e3)
    peak, punit = (peaks["hbm_gbs"], "GB/s") if w["bound"] == "hbm" else (4 * peaks["bf16_tflops"], "TFLOP/s")
    return {"metric": w["metric"], "value": round(value, 2), "unit": w["unit"], "steps": steps,
            "ms_per_step": round(ms / steps, 5), "config": w["config"]["workload"],
            "roofline": {"bound": w["bound"], "achieved": round(achieved, 2), "peak": peak, "unit": punit,
                         "frac": round(achieved / peak, 4), "traffic": profile_traffic(name), "kernel": w["kernel"]},
            "gpu_launches": w["launches_per_step"] * steps,
            "reference_gpu": reference_gpu(w, steps, warmup, dev),
            "library_gpu": reference_gpu(w, steps, warmup, dev, "library")}


# ---------------------------------------------------------------------------
def main() -> None:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    threads = len(os.sched_getaffinity(0))
    wl = args.workload

    if args.impl == "reference":
        if rank != 0:
            return
        if wl in QUANT:
            fmt, rows, k, bpe, cfg = QUANT[wl][:5]
            val, sample = cpu_quant_rate(fmt, rows, k, bpe, max(args.steps // 20, 3), min(args.warmup, 1), threads)
            unit, metric = "GB/s", f"{fmt.upper()} quant GB/s"
        elif wl == "fp4_gemm":
            val, sample = cpu_gemm_rate(threads, target_s=5.0)
            unit, metric = "TFLOP/s", "FP4 GEMM TFLOPS"
        elif wl == "nvfp4_ecdl":
            val, sample = cpu_ecdl_rate(4096, 4096, threads, target_s=5.0)
            unit, metric = "GB/s", "NVFP4 ECDL quant GB/s"
        elif wl == "nvfp4_ccdl":
            val, sample = cpu_ccdl_rate(4096, 4096, threads, target_s=5.0)
            unit, metric = "GB/s", "NVFP4 CCDL quant GB/s"
        elif wl == "nvfp4_encode_multi":
            val, sample = cpu_quant_rate("nvfp4", 4096, 4096, 2.5625, 3, 1, threads)
            unit, metric = "GB/s", "NVFP4 weight encode GB/s"
        elif wl == "nvfp4_dequant":
            val, sample = cpu_dequant_rate(threads, target_s=5.0)
            unit, metric = "GB/s", "NVFP4 dequant GB/s"
        elif wl == "nvfp4_dual":
            val, sample = cpu_dual_rate(threads, target_s=5.0)
            unit, metric = "GB/s", "NVFP4 dual encode GB/s"
        else:
            val, sample = cpu_qat_rate(wl, threads)
            unit, metric = "tokens/s", "SmolLM2 NVFP4 QAT tokens/s"
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": round(val, 4), "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "data": "synthetic", "config": {"workload": wl},
            "cpu_baseline": {"value": round(val, 4), "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        if wl.startswith("qat") and args.comm_sms > 0:
            # NCCL's kernels fit in the SMs the backward pass leaves free
            os.environ.setdefault("NCCL_MAX_CTAS", str(args.comm_sms))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    if wl in QUANT:
        w = quant_workload(wl, dev, rank)
    elif wl == "fp4_gemm":
        w = gemm_workload(dev, rank, tuple(int(v) for v in args.gemm_shape.split(",")))
    elif wl == "nvfp4_ecdl":
        w = ecdl_workload(dev, rank)
    elif wl == "nvfp4_ccdl":
        w = ccdl_workload(dev, rank)
    elif wl == "nvfp4_encode_multi":
        w = encode_multi_workload(dev, rank)
    elif wl == "nvfp4_dequant":
        w = dequant_workload(dev, rank)
    elif wl == "nvfp4_dual":
        w = dual_workload(dev, rank)
    else:
        w = qat_workload(wl, dev, rank, world, args.backend, not args.no_graph, args.comm_sms)

    def barrier():
        if world > 1:
            dist.barrier()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(int(vis.split(",")[local]) if vis else local).start()
    t_end = time.time() + args.spinup_s
    i = 0
    while time.time() < t_end and not wl.startswith("qat"):
        w["step"](i)
        i += 1
        if i % 16 == 0:
            torch.cuda.synchronize()
    for i in range(args.warmup):
        w["step"](i)
    torch.cuda.synchronize()

    run, keep = time_steps(w, args.steps, dev)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    from cdl_b200 import _lib as _cdl_lib

    launches0 = _cdl_lib.launches
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    counted_launches = _cdl_lib.launches - launches0
    if w.get("graph_launches") is not None:
        counted_launches = w["graph_launches"]() * args.steps
    ms = e0.elapsed_time(e1)
    clocks = sampler.stop()
    del keep, run
    # a bounded device-side wait that timed out in the timed steps is an error
    # (read outside the timed region)
    if w.get("check_status") is not None:
        w["check_status"]()
    else:
        _cdl_lib.check_status(dev)
    if args.torch_profile and world == 1:  # kernel breakdown, outside the timed region
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(2):
                w["step"](i)
            torch.cuda.synchronize()
        with open(args.torch_profile, "w") as f:
            f.write(prof.key_averages().table(sort_by="self_cuda_time_total", row_limit=40, max_name_column_width=90))
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = w["units_per_step"] * args.steps * world / (ms_max / 1e3)

    # end to end through the public API with host buffers
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        w["e2e_step"]()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        w["e2e_step"]()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = w["units_per_step"] * e2e_steps * world / (float(e2e_ms.item()) / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if wl in QUANT:
            fmt, rows, k, bpe, cfg = QUANT[wl][:5]
            val, sample = cpu_quant_rate(fmt, rows, k, bpe, 3, 1, threads, target_s=10.0)
        elif wl == "fp4_gemm":
            val, sample = cpu_gemm_rate(threads, target_s=10.0)
        elif wl == "nvfp4_ecdl":
            val, sample = cpu_ecdl_rate(4096, 4096, threads, target_s=10.0)
        elif wl == "nvfp4_ccdl":
            val, sample = cpu_ccdl_rate(4096, 4096, threads, target_s=10.0)
        elif wl == "nvfp4_encode_multi":
            val, sample = cpu_quant_rate("nvfp4", 4096, 4096, 2.5625, 3, 1, threads, target_s=10.0)
        elif wl == "nvfp4_dequant":
            val, sample = cpu_dequant_rate(threads, target_s=10.0)
        elif wl == "nvfp4_dual":
            val, sample = cpu_dual_rate(threads, target_s=10.0)
        else:
            val, sample = cpu_qat_rate(wl, threads)
        cpu = {"value": round(val, 4), "unit": w["unit"], "cores": threads, "kind": "port", "sample": sample}

    peaks, peak_src = load_peaks()
    per_step_s = ms_max / 1e3 / args.steps
    if w["bound"] == "hbm":
        achieved, peak, punit = w["units_per_step"] / per_step_s, peaks["hbm_gbs"], "GB/s"
    elif wl == "fp4_gemm":  # the GEMM kernel alone, A pre-quantized
        kernel_s = time_kernel(w["kernel_step"], args.steps, dev) / 1e3
        achieved, peak, punit = w["units_per_step"] / kernel_s, 4 * peaks["bf16_tflops"], "TFLOP/s"
    else:
        achieved = w["units_per_step"] * w["flops_per_unit"] / per_step_s / 1e12
        peak, punit = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), "TFLOP/s"
    line = {
        "metric": w["metric"], "value": round(value, 3), "unit": w["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": dict(w["config"], parallelism=w["config"].get("parallelism", f"replicas x{world}")),
        "roofline": {"bound": w["bound"], "achieved": round(achieved, 2), "peak": peak, "unit": punit,
                     "frac": round(achieved / peak, 4), "traffic": profile_traffic(wl),
                     "peak_source": peak_src, "kernel": w["kernel"]},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 3), "unit": w["unit"], "h2d_bytes_per_step": w["h2d"],
                "d2h_bytes_per_step": w["d2h"]},
        "gpu_launches": (counted_launches if w.get("count_launches")
                         else (w["launches_per_step"] * args.steps) if w["launches_per_step"] else None),
        "clocks": clocks,
    }
    if world == 1:  # the reference's own GPU kernels (and cuBLAS for the GEMM) on the same inputs
        for key in ("reference", "library"):
            other = reference_gpu(w, args.steps, 3, dev, key)
            if other is not None:
                line[f"{key}_gpu"] = other
    if wl == "fp4_gemm":
        line["roofline"]["peak_note"] = FP4_PEAK_NOTE
    if wl.startswith("qat"):
        line["roofline"]["peak_note"] = "model FLOPs (6P + 12 L d s per token) vs measured sustained bf16 peak"
    if world == 1 and wl.startswith("qat") and not args.no_components:
        import gc

        del w  # the QAT step's memory (its graph pool) before the component workloads
        gc.collect()
        torch.cuda.empty_cache()
        line["reference_gpu"] = reference_qat_gpu(wl, dev, min(args.steps, 10), 2)
        gc.collect()
        torch.cuda.empty_cache()
        line["components"] = {
            "nvfp4_quant": measure_component("nvfp4_quant", dev, 200, 10, peaks),
            "fp4_gemm": measure_component("fp4_gemm", dev, 20, 5, peaks),
        }
        for name in ("nvfp4_quant_large", "nvfp4_quant_t", "mxfp4_quant", "mxfp8_quant", "mxfp4_quant_t",
                     "mxfp8_quant_t", "nvfp4_encode_multi", "nvfp4_dequant", "nvfp4_dual"):
            line["components"][name] = measure_component(name, dev, 20, 3, peaks)
            torch.cuda.empty_cache()
        line["components"]["fp4_gemm"]["roofline"]["peak_note"] = FP4_PEAK_NOTE
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        # a captured step holds NCCL collectives: release it first
        if "w" in locals() and w.get("release") is not None:
            w["release"]()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
