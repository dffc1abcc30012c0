"""Block-scaled dequantize: the drop-in for ``cdl.core.kernel.dequant``.

Same functions and semantics as the reference (``cdl/core/kernel/
dequant.py:103-143``): ``bf16((value * scale) * alpha)``; ``k`` is taken from
the packed width and must be a multiple of the block.  ``block_k`` was a
Triton tiling knob and is accepted and ignored.  CUDA tensors only.
"""

from __future__ import annotations

import torch

from cdl_b200 import _lib


def _fp4_dequant(packed, scale, alpha, group_size: int, scale_is_e8m0: bool, swizzled: bool = False) -> torch.Tensor:
    dev = _lib.require_cuda(packed, scale, alpha)
    rows, half_k = packed.shape
    k = half_k * 2
    out = torch.empty((rows, k), dtype=torch.bfloat16, device=dev)
    if rows == 0 or k == 0:
        return out
    packed = packed.contiguous().view(torch.uint8)
    scale = scale.contiguous()
    alpha = alpha.reshape(-1).float().contiguous()
    _lib.call(
        "cdlb200_fp4_dequant_swizzled" if swizzled else "cdlb200_fp4_dequant", _lib.ptr(packed), _lib.ptr(scale),
        _lib.ptr(alpha), rows, k, group_size, int(scale_is_e8m0), _lib.ptr(out), _lib.stream(dev),
    )
    return out


def nvfp4_dequant(packed: torch.Tensor, scale: torch.Tensor, alpha: torch.Tensor, block_k: int = 1024, *,
                  swizzled: bool = False) -> torch.Tensor:
    """``swizzled=True``: ``scale`` is in the 128x4 GEMM layout (a B200 extension)."""
    return _fp4_dequant(packed, scale, alpha, 16, False, swizzled)


def mxfp4_dequant(packed: torch.Tensor, scale: torch.Tensor, alpha: torch.Tensor, block_k: int = 1024, *,
                  swizzled: bool = False) -> torch.Tensor:
    return _fp4_dequant(packed, scale, alpha, 32, True, swizzled)


def mxfp8_dequant(
    packed: torch.Tensor, scale: torch.Tensor, alpha: torch.Tensor | None = None, block_k: int = 1024
) -> torch.Tensor:
    dev = _lib.require_cuda(packed, scale, alpha)
    rows, k = packed.shape
    out = torch.empty((rows, k), dtype=torch.bfloat16, device=dev)
    if rows == 0 or k == 0:
        return out
    packed = packed.contiguous().view(torch.uint8)
    scale = scale.contiguous()
    a = None if alpha is None else alpha.reshape(-1).float().contiguous()
    _lib.call(
        "cdlb200_mxfp8_dequant", _lib.ptr(packed), _lib.ptr(scale), _lib.ptr(a), rows, k,
        _lib.ptr(out), _lib.stream(dev),
    )
    return out
