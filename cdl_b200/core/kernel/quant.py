"""Block-scaled quantize: the drop-in for ``cdl.core.kernel.quant``.

Same public functions, arguments, return types and errors as the reference
(``cdl/core/kernel/quant.py:126-146``):

* ``nvfp4_quant(x)`` -> ``(packed u8[rows, nb*8], scale u8[rows, nb], alpha f32[1])``
* ``mxfp4_quant(x)`` -> ``(packed u8[rows, nb*16], scale u8[rows, nb], alpha = ones(1))``
* ``mxfp8_quant(x)`` -> ``(packed e4m3[rows, nb*32], scale u8[rows, nb], None)``

raising ``ValueError`` for a non-2-D input (quant.py:79-80).  ``block_chunk``
was a Triton tiling knob and is accepted and ignored.  Two keyword extensions
serve the GEMM path: ``transpose=True`` quantizes ``x.T`` along dim 0 without
materialising the transpose (the wgrad requantize), and ``swizzled=True``
writes the scales directly in the 128x4 tiled GEMM layout.

The input is a CUDA tensor of bf16 (the tuned kernels) or fp32 / fp16 (the
reference's own fp32 arithmetic, ``cdlb200_quant_wide``), as cdl's Triton
kernel accepts any floating input; there is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch

from cdl_b200 import _lib

NVFP4, MXFP4, MXFP8 = 0, 1, 2
_BLOCK = {NVFP4: 16, MXFP4: 32, MXFP8: 32}
# input dtypes: bf16 takes the tuned kernels, fp32 / fp16 cdl's literal fp32 path
_DTYPES = {torch.bfloat16: 0, torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16}


def scale_shape(r: int, nb: int, swizzled: bool) -> tuple[int, int]:
    if swizzled:
        return ((r + 127) // 128 * 128, (nb + 3) // 4 * 4)
    return (r, nb)


def _quant(
    x: torch.Tensor, fmt: int, transpose: bool = False, swizzled: bool = False
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor [rows, k], got shape {tuple(x.shape)}")
    dev = _lib.require_cuda(x)
    if x.dtype not in _DTYPES:
        raise TypeError(f"cdl_b200 quantize takes a floating tensor (bf16, fp16, fp32), got {x.dtype}")
    if x.stride(1) != 1 or x.stride(0) < x.shape[1] or x.data_ptr() % 16:
        x = x.contiguous()
    rows, k = x.shape
    r, c = (k, rows) if transpose else (rows, k)
    B = _BLOCK[fmt]
    nb = (c + B - 1) // B
    pstride = nb * B if fmt == MXFP8 else nb * B // 2
    packed = torch.empty((r, pstride), dtype=torch.float8_e4m3fn if fmt == MXFP8 else torch.uint8, device=dev)
    scale = torch.empty(scale_shape(r, nb, swizzled), dtype=torch.uint8, device=dev)
    layout = _lib.SCALE_SWIZZLED if swizzled else _lib.SCALE_LINEAR
    ld = max(x.stride(0), 1)
    st = _lib.stream(dev)
    if x.dtype != torch.bfloat16:
        # cdl's kernel casts each block to fp32: the literal fp32 path
        alpha = torch.empty(1, dtype=torch.float32, device=dev) if fmt == NVFP4 else None
        ws = _lib.nvfp4_workspace(dev)
        _lib.call("cdlb200_quant_wide", _lib.ptr(x), _DTYPES[x.dtype], fmt, rows, k, ld, int(transpose),
                  _lib.ptr(packed), _lib.ptr(scale), layout, _lib.ptr(alpha) if alpha is not None else None,
                  _lib.ptr(ws), ws.numel(), st)
        if fmt == MXFP4:
            alpha = torch.ones(1, dtype=torch.float32, device=dev)
        return packed, scale, alpha
    if fmt == NVFP4:
        alpha = torch.empty(1, dtype=torch.float32, device=dev)
        ws = _lib.nvfp4_workspace(dev)
        _lib.call(
            "cdlb200_nvfp4_quant", _lib.ptr(x), rows, k, ld, int(transpose), _lib.ptr(packed),
            _lib.ptr(scale), layout, None, _lib.ptr(alpha), _lib.ptr(ws), ws.numel(), st,
        )
        return packed, scale, alpha
    name = "cdlb200_mxfp4_quant" if fmt == MXFP4 else "cdlb200_mxfp8_quant"
    _lib.call(name, _lib.ptr(x), rows, k, ld, int(transpose), _lib.ptr(packed), _lib.ptr(scale), layout, st)
    alpha = torch.ones(1, dtype=torch.float32, device=dev) if fmt == MXFP4 else None
    return packed, scale, alpha


def nvfp4_quant(
    x: torch.Tensor, block_chunk: int = 32, *, transpose: bool = False, swizzled: bool = False
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    packed, scale, alpha = _quant(x, NVFP4, transpose, swizzled)
    assert alpha is not None
    return packed, scale, alpha


def mxfp4_quant(
    x: torch.Tensor, block_chunk: int = 32, *, transpose: bool = False, swizzled: bool = False
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    packed, scale, alpha = _quant(x, MXFP4, transpose, swizzled)
    assert alpha is not None
    return packed, scale, alpha


def mxfp8_quant(
    x: torch.Tensor, block_chunk: int = 32, *, transpose: bool = False, swizzled: bool = False
) -> tuple[torch.Tensor, torch.Tensor, None]:
    packed, scale, _ = _quant(x, MXFP8, transpose, swizzled)
    return packed, scale, None


def nvfp4_amax(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``(gmax, alpha)`` fp32 ``[1]`` device tensors of a 2-D bf16 tensor: the
    global NVFP4 scale cdl's ``_quant`` forms (quant.py:96-101), alone."""
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor [rows, k], got shape {tuple(x.shape)}")
    dev = _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"cdl_b200 quantize takes bfloat16 input, got {x.dtype}")
    if x.stride(1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    gmax = torch.empty(1, dtype=torch.float32, device=dev)
    alpha = torch.empty(1, dtype=torch.float32, device=dev)
    ws = _lib.nvfp4_workspace(dev)
    _lib.call("cdlb200_nvfp4_amax", _lib.ptr(x), x.shape[0], x.shape[1], max(x.stride(0), 1), _lib.ptr(gmax),
              _lib.ptr(alpha), _lib.ptr(ws), ws.numel(), _lib.stream(dev))
    return gmax, alpha


def nvfp4_dual_quant(x: torch.Tensor, *, amax: torch.Tensor | None = None, gmax: torch.Tensor | None = None,
                     rows: bool = True, cols: bool = True, swizzled: bool = True):
    """NVFP4 encodings of ``x`` (blocks of 16 along dim 1) and of ``x.T``
    (blocks of 16 along dim 0) from one read of ``x``, both with the scales in
    the 128x4 GEMM layout: the same codes, scale bytes and alpha as
    ``nvfp4_quant(x, swizzled=True)`` and ``nvfp4_quant(x, transpose=True,
    swizzled=True)``.  ``x``: contiguous bf16 ``[R, C]``, R and C multiples of
    64.  The global amax is given as ``amax`` (int32 words holding bf16
    magnitude bits, e.g. a producer kernel's epilogue words) or ``gmax`` (fp32
    ``[1]``), else computed here first.  ``swizzled=False`` writes linear
    scales (``[R, C/16]`` and ``[C, R/16]``).  Returns ``(row, col)``, each
    ``(packed, scale, alpha)`` or None when not requested."""
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor [rows, k], got shape {tuple(x.shape)}")
    dev = _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"cdl_b200 quantize takes bfloat16 input, got {x.dtype}")
    r, c = x.shape
    if r % 64 or c % 64:
        raise ValueError(f"nvfp4_dual_quant needs both dimensions to be multiples of 64, got {tuple(x.shape)}")
    x = x.contiguous()
    if amax is None and gmax is None:
        gmax, _ = nvfp4_amax(x)
    alpha = torch.empty(1, dtype=torch.float32, device=dev)
    row = col = None
    t = _lib.Nvfp4DualTensor()
    t.x, t.rows, t.cols, t.alpha = x.data_ptr(), r, c, alpha.data_ptr()
    if amax is not None:
        t.amax, t.amax_words = amax.data_ptr(), amax.numel()
    else:
        t.gmax = gmax.data_ptr()
    if rows:
        row = (torch.empty(r, c // 2, dtype=torch.uint8, device=dev),
               torch.empty(scale_shape(r, c // 16, swizzled), dtype=torch.uint8, device=dev), alpha)
        t.row_packed, t.row_scale = row[0].data_ptr(), row[1].data_ptr()
    if cols:
        col = (torch.empty(c, r // 2, dtype=torch.uint8, device=dev),
               torch.empty(scale_shape(c, r // 16, swizzled), dtype=torch.uint8, device=dev), alpha)
        t.col_packed, t.col_scale = col[0].data_ptr(), col[1].data_ptr()
    if not swizzled:
        t.flags = _lib.DUAL_ROW_LINEAR | _lib.DUAL_COL_LINEAR
    _lib.call("cdlb200_nvfp4_dual_multi", ctypes.addressof(t), 1, _lib.stream(dev))
    return row, col
