"""fp32 / fp16 input to the quantizers (``cdlb200_quant_wide``) against the
oracle of cdl's fp32 arithmetic (``oracle/wide.py``): codes, scale bytes and
alpha bit-exact, row-wise and transposed, linear and 128x4 scales, ragged K,
values spanning many binades, and the bf16 path's results on bf16-valued
input."""

import numpy as np
import pytest
import torch

import oracle
from oracle.wide import quant_wide

pytestmark = pytest.mark.gpu

FMTS = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}


def _x(rows, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g) * torch.exp(2 * torch.randn(rows, 1, generator=g))
    x[0, : min(k, 16)] = 0.0  # an all-zero block
    if rows > 1 and k > 3:
        x[1, 3] = -0.0
    return x.to(dtype)


def _fn(name):
    from cdl_b200.core.kernel import quant

    return getattr(quant, f"{name}_quant")


@pytest.mark.parametrize("name", list(FMTS))
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("shape", [(64, 256), (37, 100), (300, 528), (1, 7)])
def test_wide_rowwise_matches_oracle(name, dtype, shape):
    x = _x(*shape, dtype, seed=shape[0] * 31 + shape[1])
    p, s, a = _fn(name)(x.cuda())
    rp, rs, ra = quant_wide(x.numpy(), FMTS[name])
    assert np.array_equal(p.view(torch.uint8).cpu().numpy(), rp)
    assert np.array_equal(s.cpu().numpy(), rs)
    if name == "nvfp4":
        assert a.cpu().numpy().view(np.uint32)[0] == ra.view(np.uint32)[0]
    elif name == "mxfp4":
        assert float(a) == 1.0
    else:
        assert a is None


@pytest.mark.parametrize("name", list(FMTS))
def test_wide_transposed_and_swizzled(name):
    x = _x(256, 192, torch.float32, seed=9)
    fn = _fn(name)
    p, s, _ = fn(x.cuda(), transpose=True)
    rp, rs, _ = quant_wide(x.numpy().T.copy(), FMTS[name])
    assert np.array_equal(p.view(torch.uint8).cpu().numpy(), rp)
    assert np.array_equal(s.cpu().numpy(), rs)
    p2, s2, _ = fn(x.cuda(), swizzled=True)
    rp2, rs2, _ = quant_wide(x.numpy(), FMTS[name])
    assert np.array_equal(p2.view(torch.uint8).cpu().numpy(), rp2)
    assert np.array_equal(s2.cpu().numpy(), oracle.swizzle(rs2))


@pytest.mark.parametrize("name", list(FMTS))
def test_wide_equals_bf16_path_on_bf16_values(name):
    xb = _x(512, 1024, torch.float32, seed=4).bfloat16()
    fn = _fn(name)
    want = fn(xb.cuda())
    for dtype in (torch.float32,):
        got = fn(xb.to(dtype).cuda())
        assert torch.equal(got[0].view(torch.uint8), want[0].view(torch.uint8))
        assert torch.equal(got[1], want[1])
        if want[2] is not None:
            assert torch.equal(got[2], want[2])


def test_wide_extremes_and_empty():
    from cdl_b200.core.kernel.quant import mxfp4_quant, nvfp4_quant

    x = torch.tensor([[3.0e38, -1e-40, 1e-30, 6.0] + [0.5] * 28], dtype=torch.float32)
    for name, fn in (("nvfp4", nvfp4_quant), ("mxfp4", mxfp4_quant)):
        p, s, a = fn(x.cuda())
        rp, rs, ra = quant_wide(x.numpy(), FMTS[name])
        assert np.array_equal(p.cpu().numpy(), rp) and np.array_equal(s.cpu().numpy(), rs)
    p, s, a = nvfp4_quant(torch.empty(0, 32, device="cuda"))
    assert p.shape == (0, 16) and s.shape == (0, 2)
    assert float(a) == float(np.float32(np.finfo(np.float32).tiny) * (np.float32(1) / np.float32(2688.0)))
