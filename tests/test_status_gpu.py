"""Timed-out bounded waits reach the host.

The one-launch NVFP4 quantizer waits on a grid-wide barrier for every CTA's
partial amax.  That wait is bounded: on a timeout the kernel records it in
the status word of its workspace and finishes (with a partial amax) instead
of hanging.  Here the poll limit is set to 0, so the CTAs that reach the
barrier before the last one give up at once -- a wait that runs out with
nothing faulted -- and ``check_status`` must raise, clear the word, and stay
quiet after a normal call.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_quantize_barrier_timeout_is_reported_and_cleared():
    from cdl_b200 import _lib, workloads
    from cdl_b200.core.kernel.quant import nvfp4_quant

    dev = torch.device("cuda", 0)
    x = workloads.c1_nvfp4(4096, 4096, seed=7, device="cuda")
    nvfp4_quant(x)  # workspace allocated, barrier armed
    _lib.check_status(dev)  # nothing pending
    lib = _lib.lib()
    prev = lib.cdlb200_set_wait_limit(0)
    try:
        nvfp4_quant(x)
        torch.cuda.synchronize()
    finally:
        lib.cdlb200_set_wait_limit(prev)
    with pytest.raises(_lib.CdlB200Error) as err:
        _lib.check_status(dev)
    assert err.value.status == _lib.ERR_TIMEOUT
    # cleared, and the barrier re-armed: a normal call is exact and reports nothing
    p1, s1, a1 = nvfp4_quant(x)
    p2, s2, a2 = nvfp4_quant(x)
    torch.cuda.synchronize()
    _lib.check_status(dev)
    assert torch.equal(p1, p2) and torch.equal(s1, s2) and torch.equal(a1, a2)


def test_gemm_status_word_is_clear_after_normal_calls():
    from cdl_b200 import _lib, workloads
    from cdl_b200.core.kernel.quant import nvfp4_quant
    from cdl_b200.model.wrapper.ops import mm_fp4_direct

    a, w = workloads.c3_gemm(512, 512, 1024, seed=3, device="cuda")
    ap, asf, aal = nvfp4_quant(a, swizzled=True)
    wp, wsf, wal = nvfp4_quant(w, swizzled=True)
    mm_fp4_direct(ap, wp.T, asf, wsf.T, aal * wal, 16, True)
    torch.cuda.synchronize()
    assert int(_lib.status_word(a.device).item()) == 0
    _lib.check_status(a.device)
