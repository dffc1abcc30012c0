"""Block-scaled GEMM custom ops: the drop-in for ``cdl.model.wrapper.flashinfer``.

``torch.ops.cdl_b200.mm_fp4`` and ``torch.ops.cdl_b200.mm_mxfp8`` take the same
arguments as cdl's ``cdl::mm_fp4`` / ``cdl::mm_mxfp8``
(``cdl/model/wrapper/flashinfer.py:5-62``) and return bf16 ``[M, N]``; they run
the tcgen05 block-scaled kernel of ``libcdlb200.so`` instead of FlashInfer's
sm_120-only ``b12x`` backend.  Both have fake (meta) implementations for
tracing, as in the reference.

Argument conventions (cdl's): ``a`` is the row-major operand codes ``[M, K/2]``
(FP4) or ``[M, K]`` (FP8); ``b`` is ``w_codes.T``, a ``[K', N]`` column-major
view whose storage is the row-major ``[N, K']`` weight codes; the scales are
``swizzle_scale_factors`` outputs (``b_scale`` possibly transposed, as cdl
passes ``swizzle_scale_factors(w_q).T``), flattened for FP8.

Every call passes the device's status word (``_lib.status_word``): a bounded
wait inside the GEMM that times out sets it, and ``_lib.check_status`` turns
it into an error between steps.
"""

from __future__ import annotations

import torch

from cdl_b200 import _lib


def _storage_rows(t: torch.Tensor) -> torch.Tensor:
    """Row-major [N, K'] storage behind cdl's column-major [K', N] view."""
    if t.dim() == 2 and t.t().is_contiguous():
        return t.t()
    return t.t().contiguous()


def _flat(t: torch.Tensor) -> torch.Tensor:
    """The bytes of a swizzled scale tensor in storage order."""
    if t.dim() == 2 and not t.is_contiguous() and t.t().is_contiguous():
        t = t.t()
    return t.contiguous().view(torch.uint8)


def mm_fp4_direct(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: torch.Tensor,
    b_scale: torch.Tensor,
    alpha: torch.Tensor,
    block_size: int,
    use_nvfp4: bool,
) -> torch.Tensor:
    """``mm_fp4`` without the operator dispatch (what the QLinear backends call)."""
    dev = _lib.require_cuda(a, b, a_scale, b_scale, alpha)
    a = a.contiguous().view(torch.uint8)
    brows = _storage_rows(b).view(torch.uint8)
    m, k = a.shape[0], a.shape[1] * 2
    n = brows.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    if m == 0 or n == 0:
        return out
    al = alpha.reshape(-1).float().contiguous()
    _lib.call(
        "cdlb200_mm_fp4", _lib.ptr(a), _lib.ptr(brows), _lib.ptr(_flat(a_scale)), _lib.ptr(_flat(b_scale)),
        _lib.ptr(al), m, n, k, int(block_size), int(bool(use_nvfp4)), _lib.ptr(out), n,
        _lib.ptr(_lib.status_word(dev)), _lib.stream(dev),
    )
    return out


def mm_nvfp4_alpha2(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor, b_scale: torch.Tensor,
                    alpha_a: torch.Tensor, alpha_b: torch.Tensor,
                    accumulate_into: torch.Tensor | None = None) -> torch.Tensor:
    """NVFP4 ``mm_fp4_direct`` with the two operands' alphas multiplied in the
    GEMM epilogue (``cdlb200_mm_fp4_alpha2``) instead of by a separate launch.
    With ``accumulate_into`` (a contiguous bf16 [m, n] tensor) the product is
    added to its values in the epilogue, as ``accumulate_into += product``
    would round it (``cdlb200_mm_fp4_alpha2_acc``), and that tensor is
    returned."""
    dev = _lib.require_cuda(a, b, a_scale, b_scale, alpha_a, alpha_b)
    a = a.contiguous().view(torch.uint8)
    brows = _storage_rows(b).view(torch.uint8)
    m, k = a.shape[0], a.shape[1] * 2
    n = brows.shape[0]
    if accumulate_into is not None:
        out = accumulate_into
        if (out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or not out.is_contiguous()
                or out.device != dev):
            raise ValueError("accumulate_into must be a contiguous bf16 [m, n] tensor on the operands' device")
    else:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    if m == 0 or n == 0:
        return out
    _lib.call(
        "cdlb200_mm_fp4_alpha2_acc" if accumulate_into is not None else "cdlb200_mm_fp4_alpha2",
        _lib.ptr(a), _lib.ptr(brows), _lib.ptr(_flat(a_scale)), _lib.ptr(_flat(b_scale)),
        _lib.ptr(alpha_a), _lib.ptr(alpha_b), m, n, k, 16, 1, _lib.ptr(out), n, _lib.ptr(_lib.status_word(dev)),
        _lib.stream(dev),
    )
    return out


@torch.library.custom_op("cdl_b200::mm_fp4", mutates_args=())
def mm_fp4(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: torch.Tensor,
    b_scale: torch.Tensor,
    alpha: torch.Tensor,
    block_size: int,
    use_nvfp4: bool,
) -> torch.Tensor:
    return mm_fp4_direct(a, b, a_scale, b_scale, alpha, block_size, use_nvfp4)


@mm_fp4.register_fake
def _(a, b, a_scale, b_scale, alpha, block_size, use_nvfp4):
    return torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)


def mm_mxfp8_direct(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor, b_scale: torch.Tensor) -> torch.Tensor:
    """``mm_mxfp8`` without the operator dispatch."""
    dev = _lib.require_cuda(a, b, a_scale, b_scale)
    a = a.contiguous().view(torch.uint8)
    brows = _storage_rows(b).view(torch.uint8)
    m, k = a.shape
    n = brows.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    if m == 0 or n == 0:
        return out
    _lib.call(
        "cdlb200_mm_mxfp8", _lib.ptr(a), _lib.ptr(brows), _lib.ptr(_flat(a_scale)), _lib.ptr(_flat(b_scale)),
        None, m, n, k, _lib.ptr(out), n, _lib.ptr(_lib.status_word(dev)), _lib.stream(dev),
    )
    return out


@torch.library.custom_op("cdl_b200::mm_mxfp8", mutates_args=())
def mm_mxfp8(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor, b_scale: torch.Tensor) -> torch.Tensor:
    return mm_mxfp8_direct(a, b, a_scale, b_scale)


@mm_mxfp8.register_fake
def _(a, b, a_scale, b_scale):
    return torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)
