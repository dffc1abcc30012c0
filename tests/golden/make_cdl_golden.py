"""Generate golden vectors for the CDL window, probabilities and proxy gradient.

Runs the REFERENCE's own torch formulae on CPU in fp32: the companded top-k
window and its softmax (``topk_cpmf_companded``, cdl/core/formulae.py:6-19,
with ``Format.window``, cdl/api/format.py:33-48), the proxy value, i.e. the
expected level (``topk_q_d``, formulae.py:74-83), and its autograd gradients
with respect to the input and to kappa, for the E2M1 and E4M3 level grids and
the UE4M3-without-zero and E8M0 scale grids (fp32 tables) at q = 1.
Writes ``cdl_window.npz`` beside this script: per case v, kappa, topk, the window's first index, the
probabilities, the expected level and the two gradients.

Usage: ``python tests/golden/make_cdl_golden.py --reference <path to cdl/src>``.
Needs the reference checkout; the committed outputs do not.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def values(levels: np.ndarray, seed: int) -> np.ndarray:
    """Random values over the grid plus the edges: the levels themselves,
    midpoints, zero and -0, beyond the largest level."""
    g = np.random.default_rng(seed)
    top = float(np.abs(levels).max())
    rand = g.uniform(-1.2 * top, 1.2 * top, 200).astype(np.float32)
    small = (g.standard_normal(100) * 0.5).astype(np.float32)
    mids = ((levels[1:] + levels[:-1]) / 2).astype(np.float32)
    edges = np.array([0.0, -0.0, top, -top, 2 * top, -3 * top], dtype=np.float32)
    return np.concatenate([rand, small, levels.astype(np.float32), mids, edges]).astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CDL_REFERENCE_SRC", ""))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <path to the cdl checkout's src directory>")
    sys.path.insert(0, args.reference)
    from cdl.core import formulae
    from cdl.core.format.fp4 import E2M1
    from cdl.core.format.fp8 import E4M3, E8M0, UE4M3ExcludeZero

    out = {}
    n = 0
    grids = (("e2m1", E2M1(torch.float32), (3, 5, 16)), ("e4m3", E4M3(torch.float32), (3, 5, 8)),
             ("ue4m3", UE4M3ExcludeZero(torch.float32), (3, 5)), ("e8m0", E8M0(torch.float32), (3, 5)))
    for fname, fmt, topks in grids:
        lev = fmt.level.numpy()
        for kappa in (0.5, 4.0, 20.0):
            for topk in topks:
                if fname in ("e2m1", "e4m3"):
                    vals = values(lev, 10 + n)
                else:  # scale grids: positive values over (and just beyond) the grid, levels, midpoints
                    g = np.random.default_rng(10 + n)
                    lo, hi = (-10.0, 9.5) if fname == "ue4m3" else (-100.0, 100.0)
                    inner = lev[(lev > 2.0 ** lo) & (lev < 2.0 ** hi)]
                    vals = np.concatenate([np.exp2(g.uniform(lo, hi, 200)), inner,
                                           (inner[1:] + inner[:-1]) / 2]).astype(np.float32)
                v = torch.from_numpy(vals).requires_grad_()
                k = torch.tensor(kappa, requires_grad=True)
                q = torch.ones(())
                pmf, idx = formulae.topk_cpmf_companded(v, fmt, q, k, topk)
                ev = formulae.topk_q_d(fmt.level, q, pmf, idx)
                dv, dk = torch.autograd.grad(ev.sum(), (v, k), retain_graph=True)
                # per-element d E / d kappa
                dk_el = torch.stack([torch.autograd.grad(ev[i], k, retain_graph=True)[0]
                                     for i in range(ev.numel())])
                del dk
                out.update({
                    f"c{n}_fmt": np.array(fname), f"c{n}_kappa": np.float32(kappa), f"c{n}_topk": np.int64(topk),
                    f"c{n}_v": v.detach().numpy(), f"c{n}_start": idx[:, 0].numpy().astype(np.int64),
                    f"c{n}_pmf": pmf.detach().numpy(), f"c{n}_ev": ev.detach().numpy(),
                    f"c{n}_dv": dv.numpy(), f"c{n}_dk": dk_el.numpy(),
                })
                n += 1
    out["count"] = np.int64(n)
    np.savez_compressed(os.path.join(HERE, "cdl_window.npz"), **out)
    print(f"wrote {n} cases")


if __name__ == "__main__":
    main()
