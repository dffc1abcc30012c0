"""Generate golden vectors for the CCDL eval-mode round (``cdlb200_ccdl_round``).

Runs the REFERENCE's own torch path, ``cascaded_nearest_round``
(``cdl/core/ccdl.py:78-89``) with the formats the CCDL modules build
(``E2M1`` / ``E4M3`` theta levels, ``UE4M3ExcludeZero`` / ``E8M0`` scale
levels, ``cdl/model/components/quant/ccdl/{nvfp4,mxfp4,mxfp8}.py``), on seeded
inputs, packs the indices with the formats' ``pack`` and writes
``ccdl_round.npz`` beside this script: per case the theta values (fp32 holding
values of the case's theta dtype), q, alpha, the packed codes and scale bytes,
and for bf16 levels the eval tensor's ``dequantize()`` (ccdl.py:43-48).

Usage: ``python tests/golden/make_ccdl_golden.py --reference <path to cdl/src>``.
Needs the reference checkout; the committed outputs do not.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
NVFP4, MXFP4, MXFP8 = 0, 1, 2
BLOCK = {NVFP4: 16, MXFP4: 32, MXFP8: 32}


def formats(fmt: int, dtype: torch.dtype):
    from cdl.core.format.fp4 import E2M1
    from cdl.core.format.fp8 import E4M3, E8M0, UE4M3ExcludeZero

    if fmt == NVFP4:
        return E2M1(dtype), UE4M3ExcludeZero(dtype)
    if fmt == MXFP4:
        return E2M1(dtype), E8M0(dtype)
    return E4M3(dtype), E8M0(dtype)


def case(fmt: int, theta_dtype: torch.dtype, level_dtype: torch.dtype, shared: bool, seed: int):
    from cdl.core.ccdl import cascaded_nearest_round

    g = torch.Generator().manual_seed(seed)
    B = BLOCK[fmt]
    rows, nb = 6, 5
    std = torch.exp(torch.empty(rows, 1, 1).uniform_(-3, 3, generator=g))
    theta = (torch.randn(rows, nb, B, generator=g) * std)
    theta[0, 0, :4] = torch.tensor([0.0, -0.0, 1e-30, -1e-30])
    theta[1, 1, :3] = torch.tensor([3e4, -3e4, 0.5])
    theta = theta.to(theta_dtype)
    amax = theta.float().abs().amax(dim=-1, keepdim=True)
    top = 448.0 if fmt == MXFP8 else 6.0
    jitter = torch.exp(torch.empty(rows, nb, 1).uniform_(-0.7, 0.7, generator=g))
    q = (amax / top).clamp_min(2.0 ** -126) * jitter
    q[0, 2, 0] = 1e-12  # below the smallest scale level
    q[1, 3, 0] = 1e6  # above the largest
    if shared:
        q = q[:1]
    alpha = torch.tensor(0.8371 if seed % 2 else 1.2345678)
    tf, qf = formats(fmt, level_dtype)
    ti, qi = cascaded_nearest_round(theta, tf, q, qf, alpha)
    if fmt == MXFP8:
        packed = tf.pack(ti).view(torch.uint8).reshape(rows, nb * B)
    else:
        packed = tf.pack(ti).reshape(rows, nb * B // 2)
    scale = qf.pack(qi).reshape(-1, nb).to(torch.uint8)
    out = {
        "fmt": np.int64(fmt),
        "theta": theta.float().numpy(),
        "theta_bf16": np.bool_(theta_dtype == torch.bfloat16),
        "levels_bf16": np.bool_(level_dtype == torch.bfloat16),
        "q": q.reshape(-1, nb).numpy(),
        "alpha": np.float32(alpha.item()),
        "packed": packed.numpy(),
        "scale": scale.numpy(),
    }
    if level_dtype == torch.bfloat16:
        lv = tf.level[ti.long()] * qf.level[qi.long()] * alpha.to(level_dtype)
        out["deq"] = lv.reshape(rows, nb * B).float().numpy()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CDL_REFERENCE_SRC", ""))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <path to the cdl checkout's src directory>")
    sys.path.insert(0, args.reference)
    arrays = {}
    n = 0
    for fmt in (NVFP4, MXFP4, MXFP8):
        for td in (torch.bfloat16, torch.float32):
            for ld in (torch.bfloat16, torch.float32):
                for shared in (False, True):
                    c = case(fmt, td, ld, shared, seed=100 + n)
                    for key, val in c.items():
                        arrays[f"c{n}_{key}"] = val
                    n += 1
    arrays["count"] = np.int64(n)
    np.savez_compressed(os.path.join(HERE, "ccdl_round.npz"), **arrays)
    print(f"wrote {n} cases")


if __name__ == "__main__":
    main()
