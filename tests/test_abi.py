"""CPU-side checks of the C-ABI boundary: the library loads, exports every
symbol the header declares, validates arguments on the host, and the Python
API refuses CPU tensors instead of falling back."""

import ctypes
import os
import re

import pytest
import torch

from cdl_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"\b(cdlb200_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _declared_symbols()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(lib, name), name
    assert declared <= set(_lib.SIGNATURES), declared - set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.lib()
    assert lib.cdlb200_version() >= 100
    for code in range(-7, 1):
        assert lib.cdlb200_status_string(code)
    assert lib.cdlb200_nvfp4_quant_workspace_bytes(4096, 4096) >= 256
    # the persistent kernels' SM cap: host-side setting, no GPU involved
    assert lib.cdlb200_set_persistent_sm_limit(-1) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_set_persistent_sm_limit(132) == _lib.OK
    assert lib.cdlb200_set_persistent_sm_limit(0) == _lib.OK


def test_host_side_argument_errors_need_no_gpu():
    lib = _lib.lib()
    # negative sizes, bad layout flag, bad transpose flag: rejected before any CUDA call
    assert lib.cdlb200_mxfp4_quant(None, -1, 16, 16, 0, None, None, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_mxfp8_quant(None, 4, 32, 32, 0, None, None, 7, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_mxfp8_quant(None, 4, 32, 32, 2, None, None, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_fp4_dequant(None, None, None, 4, 32, 8, 0, None, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_swizzle_scales(None, -3, 4, None, None) == _lib.ERR_INVALID_ARG
    # empty problems are valid no-ops for the MX formats
    assert lib.cdlb200_mxfp4_quant(None, 0, 16, 16, 0, None, None, 0, None) == _lib.OK
    # ld < k is invalid
    dummy = ctypes.c_void_p(16)
    # the in-place bf16 scale: n must be a multiple of 8, x 16-byte aligned
    assert lib.cdlb200_scale_bf16(dummy, 12, dummy, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_scale_bf16(ctypes.c_void_p(18), 16, dummy, None) == _lib.ERR_ALIGNMENT
    assert lib.cdlb200_scale_bf16(None, 0, None, None) == _lib.OK
    # the accumulating GEMM takes the plain GEMM's checks: block size, k % 32, ldo >= n
    assert lib.cdlb200_mm_fp4_alpha2_acc(dummy, dummy, dummy, dummy, None, None, 64, 64, 64, 32, 1, dummy, 64,
                                         None, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_mm_fp4_alpha2_acc(dummy, dummy, dummy, dummy, None, None, 64, 64, 48, 16, 1, dummy, 64,
                                         None, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_mm_fp4_alpha2_acc(dummy, dummy, dummy, dummy, None, None, 64, 64, 64, 16, 1, dummy, 32,
                                         None, None) == _lib.ERR_INVALID_ARG
    assert lib.cdlb200_mxfp4_quant(dummy, 4, 64, 32, 0, dummy, dummy, 0, None) == _lib.ERR_INVALID_ARG
    # NVFP4 needs a workspace of the stated size
    assert lib.cdlb200_nvfp4_quant(dummy, 4, 64, 64, 0, dummy, dummy, 0, None, dummy, dummy, 8, None) in (
        _lib.ERR_WORKSPACE,
    )


def test_python_api_refuses_cpu_tensors():
    from cdl_b200.core.kernel import dequant, quant

    x = torch.randn(4, 32).bfloat16()
    for fn in (quant.nvfp4_quant, quant.mxfp4_quant, quant.mxfp8_quant):
        with pytest.raises(RuntimeError, match="no CPU fallback"):
            fn(x)
    with pytest.raises(ValueError, match="2D"):
        quant.nvfp4_quant(torch.randn(2, 3, 4).bfloat16())
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        dequant.nvfp4_dequant(torch.zeros(4, 16, dtype=torch.uint8), torch.zeros(4, 2, dtype=torch.uint8), torch.ones(1))


def test_cdl_entry_points_validate_arguments_on_the_host():
    """ECDL / CCDL entry points reject bad formats, window widths, strides,
    null buffers and misalignment before touching the GPU, and treat empty
    problems as no-ops."""
    lib = _lib.lib()
    bad, ok, align = _lib.ERR_INVALID_ARG, _lib.OK, _lib.ERR_ALIGNMENT
    d = ctypes.c_void_p(256)
    # cdlb200_ccdl_round(theta, theta_f32, rows, nb, format, q, q_stride, alpha, levels_bf16, packed, scale, stream)
    assert lib.cdlb200_ccdl_round(d, 0, 4, 2, 7, d, 2, d, 1, d, d, None) == bad          # unknown format
    assert lib.cdlb200_ccdl_round(d, 0, 4, 2, 0, d, 3, d, 1, d, d, None) == bad          # q_stride not 0 / nb
    assert lib.cdlb200_ccdl_round(d, 0, -1, 2, 0, d, 2, d, 1, d, d, None) == bad         # negative rows
    assert lib.cdlb200_ccdl_round(None, 0, 4, 2, 0, d, 2, d, 1, d, d, None) == bad       # null theta
    assert lib.cdlb200_ccdl_round(ctypes.c_void_p(258), 0, 4, 2, 0, d, 2, d, 1, d, d, None) == align
    assert lib.cdlb200_ccdl_round(None, 0, 0, 2, 0, None, 2, None, 1, None, None, None) == ok  # empty
    # cdlb200_ccdl_fwd: theta window wider than the grid, q window wider than the scale grid
    assert lib.cdlb200_ccdl_fwd(d, 0, 4, 2, 0, d, 2, d, d, d, d, 17, 5, d, d, None) == bad
    assert lib.cdlb200_ccdl_fwd(d, 0, 4, 2, 0, d, 2, d, d, d, d, 5, 127, d, d, None) == bad
    # cdlb200_ecdl_fwd: unknown scale mode; topk 0
    assert lib.cdlb200_ecdl_fwd(d, 0, 4, 2, 0, 5, d, d, 5, d, d, d, d, None) == bad
    assert lib.cdlb200_ecdl_fwd(d, 0, 4, 2, 0, 0, d, d, 0, d, d, d, d, None) == bad
    # workspace sizes are host arithmetic
    assert lib.cdlb200_ccdl_bwd_workspace_bytes(0, 4, 0) == 0
    assert lib.cdlb200_ecdl_bwd_workspace_bytes(-1, 4, 0) == 0
