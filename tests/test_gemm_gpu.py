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
