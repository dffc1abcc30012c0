"""Scale-factor layout helpers: the drop-in for ``cdl.core.mm.swizzle``.

``swizzle_scale_factors`` runs a CUDA kernel (cdl/core/mm/swizzle.py:5-14:
zero-padded ``[ceil(m/128)*128, ceil(b/4)*4]`` in 128x4 tiles).  The
quantizers here can write that layout directly (``swizzled=True``), which
is what the GEMM path uses; this function serves callers that hold linear
scales.  ``expand_rows`` / ``pad_k`` / ``pad_n`` have the reference's
contract (swizzle.py:17-50: broadcast a shared scale row; zero-extend K to a
multiple; zero-extend N to a minimum and a multiple).
"""

from __future__ import annotations

import torch

from cdl_b200 import _lib


def swizzle_scale_factors(sf: torch.Tensor) -> torch.Tensor:
    dev = _lib.require_cuda(sf)
    m, b = sf.shape
    rows, cols = (m + 127) // 128 * 128, (b + 3) // 4 * 4
    out = torch.empty(rows, cols, dtype=torch.uint8, device=dev)
    if m == 0 or b == 0:
        return out.zero_()
    sf = sf.contiguous().view(torch.uint8)
    _lib.call("cdlb200_swizzle_scales", _lib.ptr(sf), m, b, _lib.ptr(out), _lib.stream(dev))
    return out


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m if m > 0 else v


def _grow(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """``t`` zero-extended to ``[rows, cols]`` (``t`` itself if it has that shape)."""
    if tuple(t.shape) == (rows, cols):
        return t
    out = t.new_zeros(rows, cols)
    out[: t.shape[0], : t.shape[1]] = t
    return out


def expand_rows(scale: torch.Tensor, rows: int) -> torch.Tensor:
    """A scale matrix whose one row is shared by every row of its operand,
    repeated for ``rows`` rows; per-row scales are returned unchanged."""
    return scale if scale.shape[0] == rows else scale.expand(rows, scale.shape[1]).contiguous()


def pad_k(packed: torch.Tensor, scale: torch.Tensor, elements_per_byte: int, block: int, multiple: int):
    """Zero-extend the reduction dimension to a multiple of ``multiple``
    elements: ``packed`` holds ``elements_per_byte`` elements per byte
    column, ``scale`` one byte per ``block`` elements (zero codes under zero
    scales add nothing to a dot product)."""
    k = packed.shape[-1] * elements_per_byte
    extra = _round_up(k, multiple) - k
    return (_grow(packed, packed.shape[0], packed.shape[1] + extra // elements_per_byte),
            _grow(scale, scale.shape[0], scale.shape[1] + extra // block))


def pad_n(packed: torch.Tensor, scale: torch.Tensor, multiple: int, minimum: int):
    """Zero-extend the rows (the GEMM's N) to ``max(rows, minimum)`` rounded
    up to a multiple of ``multiple``."""
    n = _round_up(max(packed.shape[0], minimum), multiple)
    return _grow(packed, n, packed.shape[1]), _grow(scale, n, scale.shape[1])
