"""Generate golden vectors for the quantize/dequantize parity tests.

Runs the REFERENCE's own torch path (imported from a cdl checkout) on seeded
inputs and writes the results beside this script:

* ``quant_small.npz`` -- full inputs and outputs of small and adversarial cases
  (random, outliers, K tails, exact midpoint ties, -0, all-zero blocks,
  subnormal and huge magnitudes, e8m0 byte 0, +-inf for MX);
* ``digests.json`` -- SHA-256 digests of the outputs at the benchmark sizes
  (C1 NVFP4 4096x4096; C2 MXFP4/MXFP8 [16384,2048] and [16384,8192], row-wise
  and transposed), whose inputs are regenerated from ``cdl_b200.workloads``.

The reference path (cited in the oracle header) is ``extended_nearest_round``
(``cdl/core/ecdl.py:115-131``) with fp32 format tables, packed with
``E2M1.pack`` / ``UE4M3ExcludeZero.pack`` / ``E4M3.pack`` / ``E8M0.pack``
(``cdl/core/format/fp4.py:19-21``, ``fp8.py:16-18,30-31,43-44``).  The K tail
is zero-padded first, as the reference's Triton kernel masks it with 0
(``cdl/core/kernel/quant.py:34``).  Dequantize is ``(level[t] * level[q]) *
alpha`` in fp32 then bf16, the order of ``cdl/core/kernel/dequant.py:43-47``.

Usage: ``python tests/golden/make_golden.py --reference <path to cdl/src>``.
Needs the reference checkout; the committed outputs do not.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from cdl_b200 import workloads  # noqa: E402

NVFP4, MXFP4, MXFP8 = 0, 1, 2
BLOCK = {NVFP4: 16, MXFP4: 32, MXFP8: 32}
NAMES = {NVFP4: "nvfp4", MXFP4: "mxfp4", MXFP8: "mxfp8"}


def ref_quant(x: torch.Tensor, fmt: int):
    """Reference torch path on bf16 ``x[rows, k]`` (tail zero-padded)."""
    from cdl.core.ecdl import extended_nearest_round
    from cdl.core.format.fp4 import E2M1
    from cdl.core.format.fp8 import E4M3, E8M0, UE4M3ExcludeZero

    f32 = torch.float32
    rows, k = x.shape
    B = BLOCK[fmt]
    nb = (k + B - 1) // B
    if nb * B != k:
        x = torch.nn.functional.pad(x, (0, nb * B - k))
    theta = x.reshape(rows, nb, B)
    if fmt == NVFP4:
        tf, qf, mode = E2M1(f32), UE4M3ExcludeZero(f32), "nvidia"
    elif fmt == MXFP4:
        tf, qf, mode = E2M1(f32), E8M0(f32), "ocp"
    else:
        tf, qf, mode = E4M3(f32), E8M0(f32), "ocp"
    ti, qi, gs = extended_nearest_round(theta, tf, qf, mode)
    scale = qf.pack(qi).reshape(rows, nb).to(torch.uint8)
    if fmt == MXFP8:
        packed = tf.pack(ti).view(torch.uint8).reshape(rows, nb * B)
    else:
        packed = tf.pack(ti).reshape(rows, nb * B // 2)
    # dequantize in the Triton kernel's order: (value * scale) * alpha -> bf16
    deq = (tf.level[ti.long()] * qf.level[qi.long()]).reshape(rows, nb * B)
    if fmt != MXFP8:
        deq = deq * gs.float()
    deq = deq.to(torch.bfloat16)
    alpha = gs.float().reshape(1) if fmt == NVFP4 else None
    return packed.contiguous(), scale.contiguous(), alpha, deq.contiguous()


def bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.contiguous().view(torch.uint8).numpy() if a.dtype != torch.uint8 else a.contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _bf(v) -> torch.Tensor:
    return torch.tensor(v, dtype=torch.float32).to(torch.bfloat16)


def small_cases(fmt: int) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(1234 + fmt)
    B = BLOCK[fmt]
    cases: dict[str, torch.Tensor] = {}
    cases["rand"] = workloads.c2_mx(32, 256, seed=11 + fmt)
    cases["outliers"] = workloads.c1_nvfp4(32, 256, seed=21 + fmt)
    cases["tail"] = workloads.c2_mx(19, 100, seed=31 + fmt)
    cases["tail_small"] = workloads.c2_mx(5, 7, seed=41 + fmt)
    # random finite bf16 bit patterns: every exponent range inside one block
    r = torch.randint(0, 1 << 16, (40, 8 * B), generator=g, dtype=torch.int32)
    r = torch.where((r & 0x7F80) == 0x7F80, r & 0x807F, r)  # drop inf/nan exponents
    cases["rand_bits"] = r.to(torch.int16).view(torch.bfloat16)
    # tiny magnitudes only (global amax < 2^-100): subnormal scales
    r2 = torch.randint(0, 0x0C00, (24, 4 * B), generator=g, dtype=torch.int32)
    r2 = r2 | (torch.randint(0, 2, r2.shape, generator=g, dtype=torch.int32) << 15)
    cases["tiny_bits"] = r2.to(torch.int16).view(torch.bfloat16)
    # hand-built edge rows
    rows = []
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    # exact midpoint ties at scale 1 (NVFP4: gmax=2688 -> alpha=1, block amax 6 -> s=1)
    tie = [6.0] + mids + [-m for m in mids] + [0.0] * (B - 15)
    rows.append(tie[:B] + [2688.0] + [0.0] * (B - 1))
    # MX ties: amax 6*2^e -> e8m0 scale 2^e, then exact midpoints *2^e
    for e in (-3, 0, 5):
        s = 2.0**e
        row = [6.0 * s] + [m * s for m in mids] + [-m * s for m in mids] + [0.0] * (B - 15)
        rows.append(row[:B] + [1.0] * B)
    rows.append([0.0] * B + [-0.0] * B)  # all-zero and all -0 blocks
    rows.append([1e-40, -1e-40, 3e-39] + [0.0] * (B - 3) + [2.0**-130, -(2.0**-127)] + [0.0] * (B - 2))
    rows.append([3.0e38, -3.0e38, 1.0, -1.0] + [0.5] * (B - 4) + [2.0**120] * B)
    rows.append([(-1.0) ** i * (i + 1) * 0.37 for i in range(2 * B)])
    edge = torch.stack([_bf(rw) for rw in rows])
    cases["edge"] = edge
    if fmt != NVFP4:
        inf_rows = torch.zeros(2, 2 * B)
        inf_rows[0, 3] = float("inf")
        inf_rows[0, 5] = 1.5
        inf_rows[1, B + 1] = float("-inf")
        inf_rows[1, 0] = -2.0
        cases["inf"] = inf_rows.to(torch.bfloat16)
    return cases


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CDL_REFERENCE_SRC", ""))
    ap.add_argument("--skip-big", action="store_true")
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <path to the cdl checkout's src directory>")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)

    arrays: dict[str, np.ndarray] = {}
    for fmt in (NVFP4, MXFP4, MXFP8):
        for name, x in small_cases(fmt).items():
            packed, scale, alpha, deq = ref_quant(x, fmt)
            key = f"{NAMES[fmt]}/{name}"
            arrays[key + "/x"] = bits(x)
            arrays[key + "/packed"] = packed.numpy()
            arrays[key + "/scale"] = scale.numpy()
            arrays[key + "/deq"] = bits(deq)
            if alpha is not None:
                arrays[key + "/alpha"] = alpha.numpy()
    # swizzle_scale_factors (cdl/core/mm/swizzle.py:5-14) on ragged shapes
    from cdl.core.mm.swizzle import swizzle_scale_factors

    for m, b in ((1, 1), (130, 5), (256, 8), (300, 13)):
        sf = torch.randint(0, 256, (m, b), generator=torch.Generator().manual_seed(m * 31 + b), dtype=torch.int32)
        sf = sf.to(torch.uint8)
        arrays[f"swizzle/{m}x{b}/in"] = sf.numpy()
        arrays[f"swizzle/{m}x{b}/out"] = swizzle_scale_factors(sf).contiguous().numpy()
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **arrays)

    if args.skip_big:
        return
    digests: dict[str, dict] = {}
    x = workloads.c1_nvfp4()
    packed, scale, alpha, deq = ref_quant(x, NVFP4)
    digests["c1_nvfp4_4096x4096"] = {
        "input": sha(bits(x)),
        "packed": sha(packed),
        "scale": sha(scale),
        "alpha_bits": int(alpha.view(torch.int32).item()),
        "deq": sha(bits(deq)),
    }
    for k in (2048, 8192):
        x = workloads.c2_mx(16384, k, seed=0)
        xt = x.t().contiguous()
        for fmt in (MXFP4, MXFP8):
            for tag, inp in (("rows", x), ("transposed", xt)):
                packed, scale, _, deq = ref_quant(inp, fmt)
                digests[f"c2_{NAMES[fmt]}_16384x{k}_{tag}"] = {
                    "input": sha(bits(inp)),
                    "packed": sha(packed),
                    "scale": sha(scale),
                    "deq": sha(bits(deq)),
                }
                print(f"c2 {NAMES[fmt]} {k} {tag} done", flush=True)
    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
