"""The NVFP4 quantize entry point that allocates nothing.

Some callers of this library cannot allocate device memory: a host that binds
the C ABI from another language runtime without a CUDA allocator of its own,
or a runtime that owns all device memory in a fixed arena and does not let an
operator allocate.  ``cdlb200_nvfp4_quant_noalloc`` serves them with a fixed
scratch array inside the library.  This test calls it through the C ABI and
checks it against ``cdlb200_nvfp4_quant`` (caller-provided workspace) on two
calls in a row, with different inputs so that scratch left over from the
first call would show in the second.  It runs last (file name) and passes
both on its own in a fresh process and after the other tests.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(x, transpose, layout, with_gmax):
    from cdl_b200 import _lib
    from cdl_b200.core.kernel.quant import scale_shape

    rows, k = x.shape
    r, c = (k, rows) if transpose else (rows, k)
    nb = (c + 15) // 16
    packed = torch.empty((r, nb * 8), dtype=torch.uint8, device=x.device)
    scale = torch.empty(scale_shape(r, nb, layout == _lib.SCALE_SWIZZLED), dtype=torch.uint8, device=x.device)
    gmax = torch.empty(1, dtype=torch.float32, device=x.device) if with_gmax else None
    alpha = torch.empty(1, dtype=torch.float32, device=x.device)
    return packed, scale, gmax, alpha


def _quant_with_workspace(lib, x, transpose, layout=0, with_gmax=True):
    from cdl_b200 import _lib

    rows, k = x.shape
    packed, scale, gmax, alpha = _outputs(x, transpose, layout, with_gmax)
    ws = torch.zeros(lib.cdlb200_nvfp4_quant_workspace_bytes(rows, k), dtype=torch.uint8, device=x.device)
    rc = lib.cdlb200_nvfp4_quant(x.data_ptr(), rows, k, k, int(transpose), packed.data_ptr(), scale.data_ptr(),
                                 layout, _lib.ptr(gmax), alpha.data_ptr(), ws.data_ptr(), ws.numel(),
                                 _lib.stream(x.device))
    assert rc == 0, rc
    return [t for t in (packed, scale, gmax, alpha) if t is not None]


def _quant_noalloc(lib, x, transpose, layout=0, with_gmax=True):
    from cdl_b200 import _lib

    rows, k = x.shape
    packed, scale, gmax, alpha = _outputs(x, transpose, layout, with_gmax)
    rc = lib.cdlb200_nvfp4_quant_noalloc(x.data_ptr(), rows, k, k, int(transpose), packed.data_ptr(),
                                         scale.data_ptr(), layout, _lib.ptr(gmax), alpha.data_ptr(),
                                         _lib.stream(x.device))
    assert rc == 0, rc
    return [t for t in (packed, scale, gmax, alpha) if t is not None]


def test_noalloc_matches_workspace_entry_point_two_calls():
    from cdl_b200 import _lib, workloads

    lib = _lib.lib()
    # second input has a much smaller amax, so a stale gmax/counter from the first call would show
    inputs = [workloads.c1_nvfp4(1024, 2048, seed=40).cuda(), (workloads.c2_mx(512, 1024, seed=41) * 0.01).cuda()]
    for x, transpose in zip(inputs, (False, True)):
        ref = _quant_with_workspace(lib, x, transpose)
        got = _quant_noalloc(lib, x, transpose)
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_noalloc_scratch_gmax_and_swizzled_scales():
    """No gmax output (the global amax then lives in the fixed scratch array)
    and scales in the GEMM's 128x4 layout: same packed codes, scales and
    alpha as the workspace entry point, on two calls in a row."""
    from cdl_b200 import _lib, workloads

    lib = _lib.lib()
    inputs = [workloads.c2_mx(384, 2048, seed=42).cuda(), (workloads.c1_nvfp4(256, 1024, seed=43) * 3.0).cuda()]
    for x in inputs:
        ref = _quant_with_workspace(lib, x, False, _lib.SCALE_SWIZZLED, with_gmax=False)
        got = _quant_noalloc(lib, x, False, _lib.SCALE_SWIZZLED, with_gmax=False)
        torch.cuda.synchronize()
        assert len(got) == 3
        for a, b in zip(ref, got):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_noalloc_rejects_bad_arguments():
    from cdl_b200 import _lib

    lib = _lib.lib()
    assert lib.cdlb200_nvfp4_quant_noalloc(None, -1, 16, 16, 0, None, None, 0, None, None, None) == _lib.ERR_INVALID_ARG
