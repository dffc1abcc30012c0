"""Host-side checks of the clip + AdamW entry point (no GPU needed: sizes
and argument validation run before any CUDA call)."""

import ctypes

import pytest

from cdl_b200 import _lib


def _table(numels, align=16):
    tab = (_lib.AdamwTensor * len(numels))()
    for i, n in enumerate(numels):
        base = 1 << 20 + i
        tab[i].param, tab[i].grad = base, base + 4096 * 16
        tab[i].exp_avg, tab[i].exp_avg_sq = base + 8192 * 16, base + 12288 * 16 + (align % 16)
        tab[i].numel = n
    return tab


def test_workspace_bytes_counts_chunks():
    lib = _lib.lib()
    tab = _table([8, 16384, 16392, 0, 100000])
    # 64 scalar bytes + one fp32 partial per 16384-element chunk: 1 + 1 + 2 + 0 + 7
    assert lib.cdlb200_clip_adamw_workspace_bytes(ctypes.addressof(tab), 5) == 64 + 4 * 11
    assert lib.cdlb200_clip_adamw_workspace_bytes(None, 0) == 64


@pytest.mark.parametrize("numels,align,status", [
    ([12], 16, _lib.ERR_INVALID_ARG),   # numel % 8 != 0
    ([-8], 16, _lib.ERR_INVALID_ARG),
    ([16], 4, _lib.ERR_ALIGNMENT),      # exp_avg_sq not 16-byte aligned
])
def test_argument_errors_reported_on_host(numels, align, status):
    lib = _lib.lib()
    tab = _table(numels, align)
    ws = (ctypes.c_uint8 * 1024)()
    rc = lib.cdlb200_clip_adamw(ctypes.addressof(tab), len(numels), 1.0, 1e-3, 0.9, 0.95, 1e-8, 0.0,
                                ctypes.addressof(ws), 1024, None, None)
    assert rc == status


def test_workspace_too_small():
    lib = _lib.lib()
    tab = _table([16384 * 4])
    ws = (ctypes.c_uint8 * 80)()
    rc = lib.cdlb200_clip_adamw(ctypes.addressof(tab), 1, 1.0, 1e-3, 0.9, 0.95, 1e-8, 0.0,
                                ctypes.addressof(ws), 64 + 4 * 3, None, None)
    assert rc == _lib.ERR_WORKSPACE


def test_bad_betas():
    lib = _lib.lib()
    tab = _table([16])
    ws = (ctypes.c_uint8 * 1024)()
    rc = lib.cdlb200_clip_adamw(ctypes.addressof(tab), 1, 1.0, 1e-3, 1.0, 0.95, 1e-8, 0.0,
                                ctypes.addressof(ws), 1024, None, None)
    assert rc == _lib.ERR_INVALID_ARG
