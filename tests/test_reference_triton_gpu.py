"""Parity with the reference's own GPU kernels, run on the same B200.

cdl's quantizers are Triton kernels (``cdl/core/kernel/quant.py:13-68``
``_quant_kernel``, ``dequant.py:25-72``, ``ecdl/kernel.py:12-185``
``_ecdl_fwd``, ``ccdl/kernel.py`` ``_ccdl_fwd``).  The reference package is
installed, unmodified, under ``baseline/_ref`` (git-ignored; it travels with
the working tree to the GPU box); without it these tests skip.  Each test
runs the reference kernel and the B200 kernel on the same inputs and compares
the bytes: a second parity anchor beside the CPU oracle (which restates the
reference's torch path), and for ECDL / CCDL the check that a seed draws the
reference's random stream (Triton's ``tl.rand``).

Inputs: every golden case of ``tests/golden/quant_small.npz`` (ties at each
e2m1 midpoint, -0, zero blocks, subnormal and huge magnitudes, random bf16
bit patterns, K tails), the full-size BASELINE C1 / C2 tensors, and the ECDL
/ CCDL test tensors.
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
GOLDEN = os.path.join(ROOT, "tests", "golden", "quant_small.npz")


def _ref():
    if not os.path.isdir(os.path.join(REF, "cdl")):
        pytest.skip("the reference package is not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.append(REF)
    import cdl.core.kernel.dequant as dq
    import cdl.core.kernel.quant as q

    return q, dq


def _mine():
    from cdl_b200.core.kernel import dequant, quant

    return quant, dequant


def _golden_cases(fmt):
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[1] for k in z.files if k.startswith(fmt + "/")})
    for name in names:
        yield name, torch.from_numpy(z[f"{fmt}/{name}/x"].view(np.int16)).view(torch.bfloat16)


def _same(a, b):
    a, b = a.contiguous(), b.contiguous()
    if a.dtype != torch.uint8:
        a = a.view(torch.uint8)
    if b.dtype != torch.uint8:
        b = b.view(torch.uint8)
    return a.shape == b.shape and torch.equal(a, b)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
def test_quantize_matches_reference_triton_on_golden_cases(fmt):
    """Every golden case except ``inf``: for an infinite block amax the
    reference's two paths disagree (its torch path, which the golden vectors
    and this library follow, gives E8M0 byte 254; the Triton formula
    ``floor(log2(inf)) - emax + 127`` gives 253 / 247), so that case is pinned
    by the golden vectors alone."""
    rq, _ = _ref()
    mq, _ = _mine()
    for name, x in _golden_cases(fmt):
        if name == "inf":
            continue
        xd = x.cuda()
        rp, rs, ra = getattr(rq, f"{fmt}_quant")(xd)
        mp, ms, ma = getattr(mq, f"{fmt}_quant")(xd)
        assert _same(rp, mp), (fmt, name, "codes")
        assert _same(rs, ms), (fmt, name, "scales")
        if ra is not None:
            assert torch.equal(ra.reshape(-1).cpu(), ma.reshape(-1).cpu()), (fmt, name, "alpha")


@pytest.mark.parametrize("fmt,shape,config",
                         [("nvfp4", (4096, 4096), "C1"), ("nvfp4", (16384, 8192), "C2"),
                          ("mxfp4", (16384, 8192), "C2"), ("mxfp8", (16384, 8192), "C2")],
                         ids=["nvfp4-C1", "nvfp4-C2", "mxfp4-C2", "mxfp8-C2"])
def test_quantize_matches_reference_triton_full_size(fmt, shape, config):
    """nvfp4-C2 has gmax = 47.75, for which gmax / 2688 and gmax * RN(1 / 2688)
    differ in the last bit: alpha as torch forms it on the device."""
    from cdl_b200 import workloads

    rq, rdq = _ref()
    mq, mdq = _mine()
    x = (workloads.c1_nvfp4(*shape, device="cuda") if config == "C1" else workloads.c2_mx(*shape, device="cuda"))
    rp, rs, ra = getattr(rq, f"{fmt}_quant")(x)
    mp, ms, ma = getattr(mq, f"{fmt}_quant")(x)
    assert _same(rp, mp) and _same(rs, ms)
    if ra is not None:
        assert torch.equal(ra.reshape(-1), ma.reshape(-1))
    # dequantize: both sides from the same codes
    args = (rp, rs) if fmt == "mxfp8" else (rp, rs, ra)
    rd = getattr(rdq, f"{fmt}_dequant")(*args)
    md = getattr(mdq, f"{fmt}_dequant")(*args)
    assert torch.equal(rd.view(torch.int16), md.view(torch.int16))
    # the transposed requantize (the wgrad operand) against the reference's
    # quantize of the transposed copy
    if fmt != "nvfp4" or config == "C2":
        xt = x[:, :2048]
        rp, rs, _ = getattr(rq, f"{fmt}_quant")(xt.t().contiguous())
        mp, ms, _ = getattr(mq, f"{fmt}_quant")(xt, transpose=True)
        assert _same(rp, mp) and _same(rs, ms)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_wide_input_matches_reference_triton(fmt, dtype):
    """fp32 / fp16 input, which the reference's kernel casts to fp32 per
    block: same codes, scales and alpha.  Ragged K is compared against the
    reference's torch path instead (``tests/test_quant_wide_gpu.py`` through
    ``oracle/wide.py``): for an fp32 [77, 200] NVFP4 input the reference's
    Triton kernel returned, from the ninth block of each row on, codes that
    do not encode the input under its own scale bytes, where its torch path
    and this library agree."""
    rq, _ = _ref()
    mq, _ = _mine()
    g = torch.Generator().manual_seed(5)
    for rows, k in ((512, 1024), (96, 384)):
        x = (torch.randn(rows, k, generator=g) * torch.exp(2 * torch.randn(rows, 1, generator=g))).to(dtype).cuda()
        rp, rs, ra = getattr(rq, f"{fmt}_quant")(x)
        mp, ms, ma = getattr(mq, f"{fmt}_quant")(x)
        assert _same(rp, mp) and _same(rs, ms), (rows, k)
        if ra is not None:
            assert torch.equal(ra.reshape(-1), ma.reshape(-1))


ECDL_CASES = [(0, "nvidia", 16, 4), (0, "nvidia", 16, 16), (1, "ocp", 32, 6), (2, "ocp", 32, 8)]


def _theta(m, nb, tpb, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, nb, tpb, generator=g) * torch.exp(torch.randn(m, nb, 1, generator=g))
    x[0, 0] = 0.0
    return x.bfloat16()


@pytest.mark.parametrize("fmt,mode,tpb,topk", ECDL_CASES)
def test_ecdl_forward_matches_reference_triton(fmt, mode, tpb, topk):
    """Same seed, same input: the sampled codes, scale bytes and alpha of the
    B200 ECDL kernel against the reference's ``_ecdl_fwd``."""
    _ref()
    from cdl.core.kernel.ecdl.autograd import ecdl_quant_fwd as ref_fwd
    from cdl.core.kernel.formats.spec import FormatId

    from cdl_b200.core.kernel.ecdl import ecdl_quant_fwd

    fid = [FormatId.NVFP4, FormatId.MXFP4, FormatId.MXFP8][fmt]
    theta = _theta(256, 48, tpb, 100 + fmt * 10 + topk).cuda()
    kappa = torch.tensor(3.0, device="cuda")
    for seed in (41, 12345):
        s = torch.tensor(seed, dtype=torch.int64, device="cuda")
        rp, rs, ra = ref_fwd(theta, kappa, s, int(fid), topk, mode)
        mp, ms, ma = ecdl_quant_fwd(theta, kappa, s, int(fid), topk, mode)
        assert _same(rs.reshape(-1), ms.reshape(-1))
        assert float(ra) == float(ma)
        eq = float((rp.contiguous().view(torch.uint8).reshape(-1) == mp.contiguous().view(torch.uint8).reshape(-1))
                   .float().mean())
        print(f"ecdl fmt {fmt} topk {topk} seed {seed}: codes equal {eq:.6f}")
        assert eq > 0.9999


CCDL_CASES = [(0, 16, 5, 5), (0, 16, 16, 3), (1, 32, 6, 5), (2, 32, 8, 4)]


@pytest.mark.parametrize("fmt,tpb,topk,qtopk", CCDL_CASES)
def test_ccdl_forward_matches_reference_triton(fmt, tpb, topk, qtopk):
    _ref()
    from cdl.core.kernel.ccdl.autograd import ccdl_quant_fwd as ref_fwd
    from cdl.core.kernel.formats.spec import FormatId

    from cdl_b200.core.kernel.ccdl import ccdl_quant_fwd

    fid = [FormatId.NVFP4, FormatId.MXFP4, FormatId.MXFP8][fmt]
    theta = _theta(128, 24, tpb, 200 + fmt).cuda()
    bamax = theta.float().abs().amax(-1)
    if fmt == 0:
        alpha = float(bamax.max()) / 2688.0
        q = (bamax / (6.0 * alpha)).clamp(0.01, 440.0)
    else:
        alpha = 1.0
        q = (bamax / (4.0 if fmt == 1 else 256.0)).clamp_min(1e-6)
    t = lambda v: torch.tensor(v, dtype=torch.float32, device="cuda")  # noqa: E731
    s = torch.tensor(17, dtype=torch.int64, device="cuda")
    rp, rs = ref_fwd(theta, q.float(), t(3.0), t(2.0), t(alpha), s, int(fid), topk, qtopk)
    mp, ms = ccdl_quant_fwd(theta, q.float(), t(3.0), t(2.0), t(alpha), s, int(fid), topk, qtopk)
    assert _same(rs.reshape(-1), ms.reshape(-1))
    eq = float((rp.contiguous().view(torch.uint8).reshape(-1) == mp.contiguous().view(torch.uint8).reshape(-1))
               .float().mean())
    print(f"ccdl fmt {fmt} topk {topk}/{qtopk}: codes equal {eq:.6f}")
    assert eq > 0.9999
