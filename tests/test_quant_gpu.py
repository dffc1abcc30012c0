"""GPU parity: the sm_100a quantize / dequantize kernels against the
reference's golden vectors, the oracle, and the reference's full-size
output digests."""

import hashlib

import numpy as np
import pytest
import torch

import oracle
from cdl_b200 import workloads

pytestmark = pytest.mark.gpu

FMTS = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}


def _q():
    from cdl_b200.core.kernel import quant

    return {oracle.NVFP4: quant.nvfp4_quant, oracle.MXFP4: quant.mxfp4_quant, oracle.MXFP8: quant.mxfp8_quant}


def _dq():
    from cdl_b200.core.kernel import dequant

    return {oracle.NVFP4: dequant.nvfp4_dequant, oracle.MXFP4: dequant.mxfp4_dequant, oracle.MXFP8: dequant.mxfp8_dequant}


def _to_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _np(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).cpu().numpy() if t.dtype != torch.uint8 else t.cpu().numpy()


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cases(golden):
    return sorted({k.rsplit("/", 1)[0] for k in golden.files if not k.startswith("swizzle/")})


def test_quant_matches_reference_golden(golden):
    q = _q()
    for key in _cases(golden):
        fmt = FMTS[key.split("/")[0]]
        x = _to_dev(golden[key + "/x"])
        packed, scale, alpha = q[fmt](x)
        np.testing.assert_array_equal(_np(packed), golden[key + "/packed"], err_msg=key)
        np.testing.assert_array_equal(_np(scale), golden[key + "/scale"], err_msg=key)
        if fmt == oracle.NVFP4:
            assert alpha.cpu().numpy().view(np.uint32)[0] == golden[key + "/alpha"].view(np.uint32)[0], key
        elif fmt == oracle.MXFP4:
            assert alpha.item() == 1.0
        else:
            assert alpha is None


def test_dequant_matches_reference_golden(golden):
    dq = _dq()
    for key in _cases(golden):
        fmt = FMTS[key.split("/")[0]]
        packed = torch.from_numpy(golden[key + "/packed"]).cuda()
        if fmt == oracle.MXFP8:
            packed = packed.view(torch.float8_e4m3fn)
        scale = torch.from_numpy(golden[key + "/scale"]).cuda()
        if fmt == oracle.NVFP4:
            alpha = torch.from_numpy(golden[key + "/alpha"]).cuda()
        elif fmt == oracle.MXFP4:
            alpha = torch.ones(1, device="cuda")
        else:
            alpha = None
        out = dq[fmt](packed, scale, alpha)
        np.testing.assert_array_equal(_bits(out), golden[key + "/deq"], err_msg=key)


@pytest.mark.parametrize("fmt", [oracle.NVFP4, oracle.MXFP4, oracle.MXFP8])
@pytest.mark.parametrize("shape", [(1, 32), (3, 96), (128, 512), (257, 1024), (1000, 4128), (64, 100), (7, 33)])
def test_quant_random_vs_oracle(fmt, shape):
    x = workloads.c2_mx(*shape, seed=shape[0] * 7 + shape[1] + fmt)
    xb = _bits(x)
    packed, scale, alpha = _q()[fmt](x.cuda())
    op, os_, oa = oracle.quant(xb, fmt)
    np.testing.assert_array_equal(_np(packed), op)
    np.testing.assert_array_equal(_np(scale), os_)
    if fmt == oracle.NVFP4:
        assert alpha.cpu().numpy().view(np.uint32)[0] == oa.view(np.uint32)[0]


@pytest.mark.parametrize("fmt", [oracle.NVFP4, oracle.MXFP4, oracle.MXFP8])
def test_quant_random_bit_patterns_vs_oracle(fmt):
    g = torch.Generator().manual_seed(99 + fmt)
    r = torch.randint(0, 1 << 16, (512, 1024), generator=g, dtype=torch.int32)
    r = torch.where((r & 0x7F80) == 0x7F80, r & 0x807F, r)
    xb = r.to(torch.int16).numpy().view(np.uint16)
    packed, scale, _ = _q()[fmt](_to_dev(xb))
    op, os_, _ = oracle.quant(xb, fmt)
    np.testing.assert_array_equal(_np(packed), op)
    np.testing.assert_array_equal(_np(scale), os_)


@pytest.mark.parametrize("fmt", [oracle.NVFP4, oracle.MXFP4, oracle.MXFP8])
@pytest.mark.parametrize("shape", [(64, 256), (300, 96), (33, 1000), (256, 512), (1024, 192)])
def test_transposed_quant_vs_oracle(fmt, shape):
    """Shapes with both dimensions multiples of 64 take the dual encoder's
    column pass for NVFP4 (bf16, contiguous), the others the transposing
    kernel."""
    x = workloads.c2_mx(*shape, seed=5 + fmt)
    xt_bits = _bits(x.t().contiguous())
    packed, scale, alpha = _q()[fmt](x.cuda(), transpose=True)
    op, os_, oa = oracle.quant(xt_bits, fmt)
    np.testing.assert_array_equal(_np(packed), op)
    np.testing.assert_array_equal(_np(scale), os_)


@pytest.mark.parametrize("fmt", [oracle.NVFP4, oracle.MXFP4, oracle.MXFP8])
@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("shape", [(256, 512), (130, 96), (96, 130)])
def test_swizzled_scales_vs_oracle(fmt, transpose, shape):
    x = workloads.c2_mx(*shape, seed=17 + fmt)
    src = x.t().contiguous() if transpose else x
    _, os_, _ = oracle.quant(_bits(src), fmt)
    _, scale, _ = _q()[fmt](x.cuda(), transpose=transpose, swizzled=True)
    np.testing.assert_array_equal(_np(scale), oracle.swizzle(os_))


def test_swizzle_kernel_matches_reference(golden):
    from cdl_b200.core.mm.swizzle import swizzle_scale_factors

    for key in sorted({k.rsplit("/", 1)[0] for k in golden.files if k.startswith("swizzle/")}):
        out = swizzle_scale_factors(torch.from_numpy(golden[key + "/in"]).cuda())
        np.testing.assert_array_equal(out.cpu().numpy(), golden[key + "/out"], err_msg=key)


def test_strided_input_matches_contiguous():
    x = workloads.c2_mx(64, 512, seed=3).cuda()
    view = x[:, 64:320]
    for fmt, fn in _q().items():
        a = fn(view)
        b = fn(view.contiguous())
        for u, v in zip(a, b):
            if u is not None:
                assert torch.equal(u.view(torch.uint8) if u.dtype != torch.float32 else u, v.view(torch.uint8) if v.dtype != torch.float32 else v)


def test_empty_and_errors():
    q = _q()
    e = torch.empty(0, 64, dtype=torch.bfloat16, device="cuda")
    packed, scale, alpha = q[oracle.NVFP4](e)
    assert packed.shape == (0, 32) and scale.shape == (0, 4)
    assert alpha.cpu().numpy().view(np.uint32)[0] == np.array([np.finfo(np.float32).tiny * (np.float32(1) / np.float32(2688))], np.float32).view(np.uint32)[0]
    packed, scale, alpha = q[oracle.MXFP8](torch.empty(5, 0, dtype=torch.bfloat16, device="cuda"))
    assert packed.shape == (5, 0) and scale.shape == (5, 0) and alpha is None
    with pytest.raises(ValueError):
        q[oracle.MXFP4](torch.zeros(2, 3, 4, dtype=torch.bfloat16, device="cuda"))


def test_c1_nvfp4_full_size_digest(digests):
    d = digests["c1_nvfp4_4096x4096"]
    x = workloads.c1_nvfp4()
    assert _sha(_bits(x)) == d["input"]
    packed, scale, alpha = _q()[oracle.NVFP4](x.cuda())
    assert _sha(_np(packed)) == d["packed"]
    assert _sha(_np(scale)) == d["scale"]
    assert int(alpha.cpu().numpy().view(np.int32)[0]) == d["alpha_bits"]
    deq = _dq()[oracle.NVFP4](packed, scale, alpha)
    assert _sha(_bits(deq)) == d["deq"]


@pytest.mark.parametrize("k", [2048, 8192])
def test_c2_mx_full_size_digests(digests, k):
    x = workloads.c2_mx(16384, k, seed=0)
    xd = x.cuda()
    for tag, transpose in (("rows", False), ("transposed", True)):
        for name, fmt in (("mxfp4", oracle.MXFP4), ("mxfp8", oracle.MXFP8)):
            d = digests[f"c2_{name}_16384x{k}_{tag}"]
            packed, scale, alpha = _q()[fmt](xd, transpose=transpose)
            assert _sha(_np(packed)) == d["packed"], (name, k, tag)
            assert _sha(_np(scale)) == d["scale"], (name, k, tag)
            deq = _dq()[fmt](packed, scale, alpha)
            assert _sha(_bits(deq)) == d["deq"], (name, k, tag)


def test_repeated_calls_reuse_workspace():
    x = workloads.c1_nvfp4(512, 1024, seed=9).cuda()
    first = _q()[oracle.NVFP4](x)
    for _ in range(5):
        again = _q()[oracle.NVFP4](x)
        assert all(torch.equal(a, b) for a, b in zip(first, again))
    y = x * 3
    p, s, a = _q()[oracle.NVFP4](y)
    op, os_, oa = oracle.quant(_bits(y.cpu()), oracle.NVFP4)
    np.testing.assert_array_equal(_np(p), op)
    np.testing.assert_array_equal(_np(s), os_)


def test_nvfp4_many_global_scales_vs_oracle():
    """Sweep the per-tensor scale so that many distinct block scales (and the
    encoder's rare exact patch-up and divide paths) are exercised."""
    base = workloads.c1_nvfp4(128, 1024, seed=77)
    g = torch.Generator().manual_seed(78)
    exps = torch.randint(-120, 100, (48,), generator=g).tolist()
    mants = (1.0 + torch.rand(48, generator=g)).tolist()
    for e, mnt in zip(exps, mants):
        x = (base.float() * (mnt * 2.0 ** e)).to(torch.bfloat16)
        xb = _bits(x)
        packed, scale, alpha = _q()[oracle.NVFP4](x.cuda())
        op, os_, oa = oracle.quant(xb, oracle.NVFP4)
        np.testing.assert_array_equal(_np(scale), os_, err_msg=f"scale 2^{e}*{mnt}")
        np.testing.assert_array_equal(_np(packed), op, err_msg=f"scale 2^{e}*{mnt}")
        assert alpha.cpu().numpy().view(np.uint32)[0] == oa.view(np.uint32)[0]


@pytest.mark.parametrize("fmt", [oracle.NVFP4, oracle.MXFP4])
@pytest.mark.parametrize("shape", [(128, 512), (257, 1024), (1000, 4128), (3, 96), (130, 160)])
def test_fp4_dequant_vs_oracle_linear_and_swizzled(fmt, shape):
    """The vectorized FP4 dequantize (32 elements per thread) on linear and on
    swizzled (GEMM-layout) scales: bit-identical to the oracle's dequantize."""
    x = workloads.c2_mx(*shape, seed=shape[0] + shape[1] + 31 * fmt)
    xb = _bits(x)
    op, os_, oa = oracle.quant(xb, fmt)
    want = oracle.dequant(op, os_, fmt, oa if fmt == oracle.NVFP4 else 1.0)
    packed, scale, alpha = _q()[fmt](x.cuda())
    if fmt == oracle.MXFP4:
        alpha = torch.ones(1, device="cuda")
    out = _dq()[fmt](packed, scale, alpha)
    np.testing.assert_array_equal(_bits(out), want)
    p2, s2, a2 = _q()[fmt](x.cuda(), swizzled=True)
    out2 = _dq()[fmt](p2, s2, alpha if fmt == oracle.MXFP4 else a2, swizzled=True)
    np.testing.assert_array_equal(_bits(out2), want)
