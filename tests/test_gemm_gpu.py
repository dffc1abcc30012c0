"""GPU parity of the tcgen05 block-scaled GEMMs against the fp32
dequantize-then-matmul oracle (the definition of cdl's mm_fp4 / mm_mxfp8)."""

import numpy as np
import pytest
import torch

import oracle
from cdl_b200 import workloads

pytestmark = pytest.mark.gpu

FMT = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _run(fmt_name, m, n, k, seed=0):
    from cdl_b200.core.kernel import quant
    from cdl_b200.core.mm.swizzle import swizzle_scale_factors
    from cdl_b200.model.wrapper.ops import mm_fp4, mm_mxfp8

    a, w = workloads.c3_gemm(m, n, k, seed=seed)
    qf = {"nvfp4": quant.nvfp4_quant, "mxfp4": quant.mxfp4_quant, "mxfp8": quant.mxfp8_quant}[fmt_name]
    ap, asf, aal = qf(a.cuda())
    wp, wsf, wal = qf(w.cuda())
    if fmt_name == "mxfp8":
        out = mm_mxfp8(ap, wp.T, swizzle_scale_factors(asf).flatten(), swizzle_scale_factors(wsf).flatten())
        alpha = 1.0
    else:
        alpha_t = aal * wal
        out = mm_fp4(ap, wp.T, swizzle_scale_factors(asf), swizzle_scale_factors(wsf).T, alpha_t,
                     16 if fmt_name == "nvfp4" else 32, fmt_name == "nvfp4")
        alpha = float(alpha_t.item())
    ref = oracle.mm(ap.view(torch.uint8).cpu().numpy(), asf.cpu().numpy(), wp.view(torch.uint8).cpu().numpy(),
                    wsf.cpu().numpy(), FMT[fmt_name], alpha)
    return out.float().cpu().numpy(), ref


def _rel_l2(x, y):
    return float(np.linalg.norm(x - y) / max(np.linalg.norm(y), 1e-30))


@pytest.mark.parametrize("fmt_name", ["nvfp4", "mxfp4", "mxfp8"])
@pytest.mark.parametrize("shape", [(128, 128, 256), (256, 384, 512), (200, 136, 576), (512, 1024, 2048),
                                   (384, 520, 1088), (64, 300, 4096), (1000, 2048, 1024),
                                   (2300, 2600, 320)])
def test_gemm_vs_oracle(fmt_name, shape):
    got, ref = _run(fmt_name, *shape)
    ref_bf16 = torch.from_numpy(ref).bfloat16().float().numpy()
    # the kernel rounds its fp32 accumulator to bf16, as cdl's op returns bf16
    assert _rel_l2(got, ref_bf16) <= 1e-3, _rel_l2(got, ref_bf16)
    assert _rel_l2(got, ref) <= 3e-3, _rel_l2(got, ref)


def _sample_rows(m: int, rng: np.random.Generator) -> np.ndarray:
    """Every row of two whole 256-row output tiles (the first and a random
    one) plus 96 random rows: covers whole tiles, tile edges and the last
    (possibly ragged) row block."""
    tiles = {0, int(rng.integers(0, (m + 255) // 256))}
    rows = {r for t in tiles for r in range(256 * t, min(256 * t + 256, m))}
    rows |= {int(r) for r in rng.integers(0, m, 96)} | {m - 1}
    return np.array(sorted(rows))


# 8192^3 and the shape sweep, plus a long-K case in which
# the persistent kernel's K pipeline wraps its stage ring many times
C3_PARITY_SHAPES = workloads.C3_SHAPES + [(256, 256, 16384)]


@pytest.mark.parametrize("fmt_name", ["nvfp4", "mxfp4", "mxfp8"])
@pytest.mark.parametrize("shape", C3_PARITY_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_c3_shapes_vs_oracle(fmt_name, shape):
    """Full GEMM on the GPU; the fp32 oracle on a row sample of the output.

    Tolerances (the contract is the fp32 dequantize-then-matmul oracle):
    rel-L2 <= 1e-3 against the oracle rounded to bf16 -- the kernel's output
    is bf16, whose rounding alone is ~1.1e-3 rel-L2 against unrounded fp32 --
    and <= 3e-3 against fp32; elementwise |got - ref| <= 2^-7 |ref| (one bf16
    ulp: the fp32 accumulation order may move a value across a bf16 rounding
    boundary) + 1e-4 * rms(ref row)."""
    from cdl_b200.core.kernel import quant
    from cdl_b200.model.wrapper.ops import mm_fp4_direct, mm_mxfp8_direct

    m, n, k = shape
    a, w = workloads.c3_gemm(m, n, k, seed=5, device="cuda")
    qf = {"nvfp4": quant.nvfp4_quant, "mxfp4": quant.mxfp4_quant, "mxfp8": quant.mxfp8_quant}[fmt_name]
    ap, asf, aal = qf(a, swizzled=True)
    wp, wsf, wal = qf(w, swizzled=True)
    if fmt_name == "mxfp8":
        out = mm_mxfp8_direct(ap, wp.T, asf.flatten(), wsf.flatten())
        alpha = 1.0
    else:
        alpha_t = aal * wal
        out = mm_fp4_direct(ap, wp.T, asf, wsf.T, alpha_t, 16 if fmt_name == "nvfp4" else 32,
                            fmt_name == "nvfp4")
        alpha = float(alpha_t.item())
    rows = _sample_rows(m, np.random.default_rng(m * 7 + n * 3 + k))
    rows_t = torch.from_numpy(rows).cuda()
    got = out[rows_t].float().cpu().numpy()
    # linear scales of the same operands (same bytes, other layout) for the oracle
    a_lin = qf(a)
    w_lin = qf(w)
    ap_s = a_lin[0].view(torch.uint8)[rows_t].cpu().numpy()
    as_s = a_lin[1][rows_t].cpu().numpy()
    ref = oracle.mm(ap_s, as_s, w_lin[0].view(torch.uint8).cpu().numpy(), w_lin[1].cpu().numpy(), FMT[fmt_name],
                    alpha)
    del out
    ref_bf16 = torch.from_numpy(ref).bfloat16().float().numpy()
    assert _rel_l2(got, ref_bf16) <= 1e-3, _rel_l2(got, ref_bf16)
    assert _rel_l2(got, ref) <= 3e-3, _rel_l2(got, ref)
    row_rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2, axis=1, keepdims=True))
    bound = 2.0 ** -7 * np.abs(ref) + 1e-4 * row_rms
    bad = np.abs(got - ref) > bound
    assert not bad.any(), (int(bad.sum()), np.argwhere(bad)[:5])


@pytest.mark.parametrize("shape", [(256, 512, 256), (200, 384, 320), (1000, 2048, 1024), (520, 576, 192),
                                   (130, 96, 64), (64, 200, 128), (300, 136, 576)],
                         ids=lambda s: "x".join(map(str, s)))
def test_gemm_accumulate_matches_torch_add(shape):
    """``cdlb200_mm_fp4_alpha2_acc`` (the dgrad GEMM that adds into the input
    gradient another linear already wrote) equals the plain GEMM followed by
    torch's bf16 add, bit for bit: the pair kernel (N a multiple of 64; 576
    ends in a half-filled tile), the single-CTA kernel (N <= 128, or N not a
    multiple of 64) and its ragged-column path (N = 200, 136)."""
    from cdl_b200.core.kernel import quant
    from cdl_b200.core.mm.swizzle import swizzle_scale_factors
    from cdl_b200.model.wrapper.ops import mm_nvfp4_alpha2

    m, n, k = shape
    a, w = workloads.c3_gemm(m, n, k, seed=5)
    ap, asf, aal = quant.nvfp4_quant(a.cuda())
    wp, wsf, wal = quant.nvfp4_quant(w.cuda())
    args = (ap, wp.T, swizzle_scale_factors(asf), swizzle_scale_factors(wsf).T, aal, wal)
    prior = torch.randn(m, n, generator=torch.Generator().manual_seed(1)).bfloat16().cuda()
    prior[0, 0] = 0.0
    prod = mm_nvfp4_alpha2(*args)
    want = prior + prod
    buf = prior.clone()
    got = mm_nvfp4_alpha2(*args, accumulate_into=buf)
    assert got.data_ptr() == buf.data_ptr()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # a second accumulation adds on top, in the order autograd would add
    mm_nvfp4_alpha2(*args, accumulate_into=buf)
    assert torch.equal(buf.view(torch.int16), (want + prod).view(torch.int16))
