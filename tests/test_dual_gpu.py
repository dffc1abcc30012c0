"""GPU parity of the dual NVFP4 encoder (x and x^T from one read of x, the
operands of the quantized dgrad / wgrad GEMMs) against the CPU oracle and
against the single-direction quantizers (themselves pinned to the reference's
golden vectors): codes, GEMM-layout scale bytes and alpha bit for bit."""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from cdl_b200 import workloads

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _oracle_swizzled(x_bits):
    p, s, a = oracle.quant(x_bits, oracle.NVFP4)
    return p, oracle.swizzle(s), a


@pytest.mark.parametrize("shape", [(64, 64), (128, 576), (576, 192), (192, 1536), (320, 2048)])
def test_dual_vs_oracle(shape):
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant

    x = workloads.c1_nvfp4(*shape, seed=sum(shape))
    row, col = nvfp4_dual_quant(x.cuda())
    torch.cuda.synchronize()
    b = _bits(x)
    p, s, a = _oracle_swizzled(b)
    pt, st, at = _oracle_swizzled(np.ascontiguousarray(b.T))
    assert np.array_equal(row[0].cpu().numpy(), p)
    assert np.array_equal(row[1].cpu().numpy(), s)
    assert np.array_equal(col[0].cpu().numpy(), pt)
    assert np.array_equal(col[1].cpu().numpy(), st)
    assert row[2].cpu().numpy().view(np.uint32)[0] == a.view(np.uint32)[0] == at.view(np.uint32)[0]


@pytest.mark.parametrize("shape", [(8192, 2048), (2048, 8192), (16384, 576)])
def test_dual_matches_single_direction_quantizers(shape):
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant, nvfp4_quant

    x = workloads.c2_mx(*shape, seed=3, device="cuda")
    row, col = nvfp4_dual_quant(x)
    rp, rs, ra = nvfp4_quant(x, swizzled=True)
    # x^T's encoding by the row-wise quantizer of the transposed copy (the
    # library's own transposed quantize runs the dual encoder for these shapes)
    cp, cs, ca = nvfp4_quant(x.t().contiguous(), swizzled=True)
    torch.cuda.synchronize()
    assert torch.equal(row[0], rp) and torch.equal(row[1], rs) and torch.equal(row[2], ra)
    assert torch.equal(col[0], cp) and torch.equal(col[1], cs) and torch.equal(col[2], ca)
    # the same with linear scale layouts
    lrow, lcol = nvfp4_dual_quant(x, swizzled=False)
    lp, ls, _ = nvfp4_quant(x)
    tp, ts, _ = nvfp4_quant(x.t().contiguous())
    assert torch.equal(lrow[0], lp) and torch.equal(lrow[1], ls)
    assert torch.equal(lcol[0], tp) and torch.equal(lcol[1], ts)


def test_dual_with_amax_words_and_one_direction():
    """The producer-epilogue form of the amax (bf16 magnitude bits in several
    words) gives the same result; a direction can be left out."""
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant

    x = workloads.c1_nvfp4(256, 320, seed=9, device="cuda")
    mag = int(x.abs().max().view(torch.int16).item()) & 0x7FFF
    words = torch.zeros(32, dtype=torch.int32, device="cuda")
    words[5] = mag
    words[17] = mag // 2
    ref_row, ref_col = nvfp4_dual_quant(x)
    row, none = nvfp4_dual_quant(x, amax=words, cols=False)
    none2, col = nvfp4_dual_quant(x, amax=words, rows=False)
    torch.cuda.synchronize()
    assert none is None and none2 is None
    for a, b in zip(ref_row, row):
        assert torch.equal(a, b)
    for a, b in zip(ref_col, col):
        assert torch.equal(a, b)


def test_dual_multi_tensor_launch():
    """Several tensors of different shapes and amax in one launch."""
    from cdl_b200 import _lib
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant, scale_shape

    xs = [workloads.c1_nvfp4(r, c, seed=i, device="cuda") * (10.0 ** (i - 1)) for i, (r, c) in
          enumerate([(128, 192), (576, 64), (64, 1024)])]
    gm = [torch.tensor([float(x.abs().max())], device="cuda") for x in xs]
    table = (_lib.Nvfp4DualTensor * len(xs))()
    outs = []
    for t, x, g in zip(table, xs, gm):
        r, c = x.shape
        o = [torch.empty(r, c // 2, dtype=torch.uint8, device="cuda"),
             torch.empty(scale_shape(r, c // 16, True), dtype=torch.uint8, device="cuda"),
             torch.empty(c, r // 2, dtype=torch.uint8, device="cuda"),
             torch.empty(scale_shape(c, r // 16, True), dtype=torch.uint8, device="cuda"),
             torch.empty(1, dtype=torch.float32, device="cuda")]
        outs.append(o)
        t.x, t.rows, t.cols, t.gmax, t.alpha = x.data_ptr(), r, c, g.data_ptr(), o[4].data_ptr()
        t.row_packed, t.row_scale, t.col_packed, t.col_scale = (o[0].data_ptr(), o[1].data_ptr(), o[2].data_ptr(),
                                                                o[3].data_ptr())
    _lib.call("cdlb200_nvfp4_dual_multi", ctypes.addressof(table), len(xs), _lib.stream(xs[0].device))
    for x, o in zip(xs, outs):
        row, col = nvfp4_dual_quant(x)
        torch.cuda.synchronize()
        assert torch.equal(o[0], row[0]) and torch.equal(o[1], row[1]) and torch.equal(o[4], row[2])
        assert torch.equal(o[2], col[0]) and torch.equal(o[3], col[1])


def test_dual_rejects_ragged_shapes():
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant

    with pytest.raises(ValueError):
        nvfp4_dual_quant(torch.zeros(96, 64, dtype=torch.bfloat16, device="cuda"))
