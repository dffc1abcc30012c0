"""Scale-factor layout helpers: the drop-in for ``cdl.core.mm.swizzle``.

``swizzle_scale_factors`` runs a CUDA kernel (cdl/core/mm/swizzle.py:5-14:
zero-padded ``[ceil(m/128)*128, ceil(b/4)*4]`` in 128x4 tiles).  The
quantizers here can write that layout directly (``swizzled=True``), which
is what the GEMM path uses; this function serves callers that hold linear
scales.  ``expand_rows`` / ``pad_k`` / ``pad_n`` keep the reference's
semantics (swizzle.py:17-50) and are plain tensor reshapes.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

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


def expand_rows(scale: torch.Tensor, rows: int) -> torch.Tensor:
    if scale.shape[0] != rows:
        scale = scale.expand(rows, -1).contiguous()
    return scale


def pad_k(packed: torch.Tensor, scale: torch.Tensor, elements_per_byte: int, block: int, multiple: int):
    k = packed.shape[-1] * elements_per_byte
    pad = -k % multiple
    if pad:
        packed = F.pad(packed, (0, pad // elements_per_byte))
        scale = F.pad(scale, (0, pad // block))
    return packed, scale


def pad_n(packed: torch.Tensor, scale: torch.Tensor, multiple: int, minimum: int):
    target = max(packed.shape[0], minimum)
    target += -target % multiple
    n_pad = target - packed.shape[0]
    if n_pad:
        packed = F.pad(packed, (0, 0, 0, n_pad))
        scale = F.pad(scale, (0, 0, 0, n_pad))
    return packed, scale
