"""Block-scaled matmul with the STE, shared by the ``nvfp4`` / ``mxfp4`` /
``mxfp8`` backends (cdl/core/mm/nvfp4.py:9-63, mxfp4.py:9-63, mxfp8.py:9-70).

Forward: both operands are quantized by the B200 kernels, their scales
swizzled into the 128x4 GEMM layout, and the tcgen05 block-scaled GEMM
produces bf16 ``alpha * deq(x) @ deq(w)^T`` (MXFP8 applies alpha outside the
GEMM, as cdl does).

Backward, two variants (the straight-through estimator in both: gradients
flow to the unquantized proxies):

* reference numerics (backends ``nvfp4`` / ``mxfp4`` / ``mxfp8``), as cdl:
  ``dx = g @ deq(w)``, ``dw = g^T @ deq(x)`` with bf16 operands;
* quantized backward (backends ``*_qbwd``): the dgrad and wgrad GEMMs run in
  the same block-scaled format on the tensor cores --
  ``dx = Q(g) . Q(w^T)^T`` (both quantized along N) and
  ``dw = Q(g^T) . Q(x^T)^T`` (both quantized along M, the transposed
  requantize) -- so all three GEMMs of a linear layer are FP4 (FP8).  For
  NVFP4 with every dimension a multiple of 64 each operand is read once for
  both of its encodings (``nvfp4_dual_quant``): x and w in the forward (the
  weights by the optimizer's encoder when it ran), g in the backward.
"""

from __future__ import annotations

import weakref

import torch

from cdl_b200.api.quant import QTensor
from cdl_b200.core.kernel.dequant import mxfp4_dequant, mxfp8_dequant, nvfp4_dequant
from cdl_b200.core.kernel.quant import mxfp4_quant, mxfp8_quant, nvfp4_dual_quant, nvfp4_quant
from cdl_b200.core.mm.swizzle import expand_rows, pad_k, pad_n, swizzle_scale_factors
from cdl_b200.model.components.fused import grad_amax
from cdl_b200.model.wrapper.ops import mm_fp4_direct as mm_fp4
from cdl_b200.model.wrapper.ops import mm_mxfp8_direct as mm_mxfp8
from cdl_b200.model.wrapper.ops import mm_nvfp4_alpha2

_DEQ = {"nvfp4": nvfp4_dequant, "mxfp4": mxfp4_dequant, "mxfp8": mxfp8_dequant}
_QUANT = {"nvfp4": nvfp4_quant, "mxfp4": mxfp4_quant, "mxfp8": mxfp8_quant}


def _qmm(fmt: str, a, b) -> torch.Tensor:
    """``alpha * deq(a) @ deq(b)^T`` for two ``(codes, swizzled scales, alpha)``
    triples quantized along their common last dimension."""
    (ap, asf, aal), (bp, bsf, bal) = a, b
    if fmt == "mxfp8":
        return mm_mxfp8(ap.view(torch.uint8), bp.view(torch.uint8).T, asf.flatten(), bsf.flatten())
    return mm_fp4(ap, bp.T, asf, bsf.T, aal * bal, 16 if fmt == "nvfp4" else 32, fmt == "nvfp4")


def _quantized_grads(fmt: str, g: torch.Tensor, x: torch.Tensor | None, w: torch.Tensor | None):
    """dgrad / wgrad of ``g = d(x @ w^T)`` with both GEMMs in ``fmt``."""
    q = _QUANT[fmt]
    dx = dw = None
    if w is not None:  # [M, N] x [N, K]: reduce over N
        dx = _qmm(fmt, q(g, swizzled=True), q(w, transpose=True, swizzled=True))
    if x is not None:  # [N, M] x [M, K]: reduce over M
        dw = _qmm(fmt, q(g, transpose=True, swizzled=True), q(x, transpose=True, swizzled=True))
    return dx, dw


# dequantized activations of recent backward calls, most recent first: the
# linears that share an input (q/k/v, gate/up) share its codes tensor, so its
# backward dequantize runs once
_DEQUANTIZED: list = []


def _dequant_activation(deq, codes, scales, alpha, kw):
    key = (codes.data_ptr(), codes._version, scales.data_ptr(), bool(kw))
    for ref, k, out in _DEQUANTIZED:
        if k == key and ref() is codes:
            return out
    out = deq(codes, scales, alpha, **kw)
    _DEQUANTIZED.insert(0, (weakref.ref(codes), key, out))
    del _DEQUANTIZED[2:]
    return out


# The input gradient of the quantized linears that read one input (q / k / v,
# gate / up: their activations share one dual encoding, so one codes tensor)
# is formed in one buffer: the first dgrad GEMM of the backward pass writes
# it and returns it to autograd; the others add their product to it in their
# epilogue (bf16(product) + buffer, rounded as autograd's add of the two
# gradients) and return None, so autograd adds nothing more.  Autograd runs
# the node that consumes the sum only after all of them, and the buffer
# reaches it by reference (QLinear's 2-D view of a contiguous input).
FUSE_DGRAD_SUM = True
_DGRAD_SUM_ATTR = "_cdlb200_dgrad_sum"
dgrad_accumulates = 0  # dgrad GEMMs that added into another linear's (diagnostic count)


class _DgradSum:
    __slots__ = ("users", "done", "buf")

    def __init__(self):
        self.users = 0  # forward calls that need this input's gradient
        self.done = 0   # dgrad GEMMs of the backward pass so far
        self.buf = None


def _join_dgrad_sum(codes: torch.Tensor) -> _DgradSum:
    share = getattr(codes, _DGRAD_SUM_ATTR, None)
    if share is None or share.done > 0:  # none yet, or one whose backward has begun
        share = _DgradSum()
        setattr(codes, _DGRAD_SUM_ATTR, share)
    share.users += 1
    return share


class BlockScaledMatMul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fmt: str, x: QTensor, x_proxy, w: QTensor, w_proxy, quantized_backward: bool = False):
        ctx.fmt = fmt
        ctx.swizzled = False
        ctx.dual = False
        if (quantized_backward and fmt == "nvfp4" and x_proxy is not None and w_proxy is not None
                and hasattr(x, "encode_dual") and hasattr(w, "encode_dual") and x.k == w.k
                and all(d % 64 == 0 for d in (x_proxy.numel() // x.k, x.k, w.theta.shape[0]))):
            # NVFP4 forward and quantized backward from dual encodings: x and w
            # each read once for their operand of this GEMM and the transposed
            # one of the wgrad / dgrad GEMM
            (x_row, x_col), (w_row, w_col) = x.encode_dual(), w.encode_dual()
            ctx.dual = True
            ctx.save_for_backward(*x_col, *w_col)
            ctx.share = _join_dgrad_sum(x_row[0]) if FUSE_DGRAD_SUM and x_proxy.requires_grad else None
            return mm_nvfp4_alpha2(x_row[0], w_row[0].T, x_row[1], w_row[1].T, x_row[2], w_row[2])
        # the quantized backward needs every GEMM dimension to be a multiple of 32
        ctx.qbwd = bool(quantized_backward) and x_proxy is not None and w_proxy is not None and all(
            d % 32 == 0 for d in (*x_proxy.shape, w_proxy.shape[0]))
        if ctx.qbwd:
            ctx.proxies = (x_proxy.reshape(-1, x_proxy.shape[-1]), w_proxy)
        ctx.x_k = x_proxy.shape[-1] if x_proxy is not None else None
        ctx.w_k = w_proxy.shape[-1] if w_proxy is not None else None
        if (fmt != "mxfp8" and hasattr(x, "encode_swizzled") and hasattr(w, "encode_swizzled")
                and x.k == w.k and x.k % 32 == 0 and w.theta.shape[0] % 8 == 0):
            # codes and GEMM-layout scales from one quantize launch per operand;
            # the backward dequantizes from the same swizzled scales
            x_theta, x_q, x_alpha = x.encode_swizzled(fmt)
            w_theta, w_q, w_alpha = w.encode_swizzled(fmt)
            if not ctx.qbwd:
                ctx.swizzled = True
                # dequantized copies formed with the encodings, where there are
                # some, replace the backward's dequantize
                x_deq = x.cached_dequant(fmt) if hasattr(x, "cached_dequant") else None
                w_deq = w.cached_dequant(fmt) if hasattr(w, "cached_dequant") else None
                ctx.x_deq, ctx.w_deq = x_deq is not None, w_deq is not None
                ctx.save_for_backward(*([x_deq] if ctx.x_deq else [x_theta, x_q, x_alpha]),
                                      *([w_deq] if ctx.w_deq else [w_theta, w_q, w_alpha]))
            return mm_fp4(x_theta, w_theta.T, x_q, w_q.T, x_alpha * w_alpha, 16 if fmt == "nvfp4" else 32,
                          fmt == "nvfp4")
        x_theta, x_q, x_alpha = getattr(x, fmt)()
        w_theta, w_q, w_alpha = getattr(w, fmt)()
        x_theta = x_theta.reshape(-1, x_theta.shape[-1])
        x_q = expand_rows(x_q.reshape(-1, x_q.shape[-1]), x_theta.shape[0])
        if fmt == "mxfp8":
            x_theta, x_q = pad_k(x_theta.view(torch.uint8), x_q, 1, 32, 128)
            w_theta, w_q = pad_k(w_theta.view(torch.uint8), w_q, 1, 32, 128)
        else:
            block = 16 if fmt == "nvfp4" else 32
            x_theta, x_q = pad_k(x_theta, x_q, 2, block, 32)
            w_theta, w_q = pad_k(w_theta, w_q, 2, block, 32)
        if not ctx.qbwd:  # the quantized backward requantizes the proxies instead
            ctx.save_for_backward(x_theta, x_q, x_alpha, w_theta, w_q, w_alpha)
        n = w_theta.shape[0]
        w_theta, w_q = pad_n(w_theta, w_q, 8, 128 if fmt == "mxfp8" else 0)
        if fmt == "mxfp8":
            out = mm_mxfp8(x_theta, w_theta.T, swizzle_scale_factors(x_q).flatten(),
                           swizzle_scale_factors(w_q).flatten())[:, :n]
            if x_alpha is None and w_alpha is None:
                return out
            scale = w_alpha if x_alpha is None else (x_alpha if w_alpha is None else x_alpha * w_alpha)
            return (out.float() * scale).to(torch.bfloat16)
        return mm_fp4(x_theta, w_theta.T, swizzle_scale_factors(x_q), swizzle_scale_factors(w_q).T,
                      x_alpha * w_alpha, 16 if fmt == "nvfp4" else 32, fmt == "nvfp4")[:, :n]

    @staticmethod
    def backward(ctx, grad_output):
        grad_output = grad_output.contiguous()
        if ctx.dual:
            # dx = Q(g) . Q(w^T)^T (both along N), dw = Q(g^T) . Q(x^T)^T (both
            # along M); g is read once for both of its encodings
            xc_p, xc_s, xc_a, wc_p, wc_s, wc_a = ctx.saved_tensors
            need_dx, need_dw = ctx.needs_input_grad[2], ctx.needs_input_grad[4]
            g2 = grad_output.reshape(-1, grad_output.shape[-1])
            g_row, g_col = nvfp4_dual_quant(g2, amax=grad_amax(g2), rows=need_dx, cols=need_dw)
            dx = None
            if need_dx:
                share = ctx.share
                if share is not None and share.buf is not None:  # add to the first linear's dgrad
                    global dgrad_accumulates
                    mm_nvfp4_alpha2(g_row[0], wc_p.T, g_row[1], wc_s.T, g_row[2], wc_a, accumulate_into=share.buf)
                    dgrad_accumulates += 1
                    share.done += 1
                    if share.done == share.users:
                        share.buf = None
                else:
                    dx = mm_nvfp4_alpha2(g_row[0], wc_p.T, g_row[1], wc_s.T, g_row[2], wc_a)
                    if share is not None:
                        share.done += 1
                        if share.users > 1:
                            share.buf = dx
            dw = mm_nvfp4_alpha2(g_col[0], xc_p.T, g_col[1], xc_s.T, g_col[2], xc_a) if need_dw else None
            return None, None, dx, None, dw, None
        if ctx.qbwd:
            x_src, w_src = ctx.proxies
            dx, dw = _quantized_grads(ctx.fmt, grad_output, x_src if ctx.w_k is not None else None,
                                      w_src if ctx.x_k is not None else None)
            return None, None, dx, None, dw, None
        if ctx.swizzled:
            saved = list(ctx.saved_tensors)
            x_deq = saved.pop(0) if ctx.x_deq else None
            if x_deq is None:
                x_theta, x_q, x_alpha = saved[:3]
                saved = saved[3:]
            w_deq = saved[0] if ctx.w_deq else None
            if w_deq is None:
                w_theta, w_q, w_alpha = saved
            deq = _DEQ[ctx.fmt]
            dx = dw = None
            if ctx.x_k is not None:
                if w_deq is None:
                    w_deq = deq(w_theta, w_q, w_alpha, swizzled=True)
                dx = grad_output @ w_deq[:, : ctx.x_k]
            if ctx.w_k is not None:
                if x_deq is None:
                    x_deq = _dequant_activation(deq, x_theta, x_q, x_alpha, {"swizzled": True})
                dw = grad_output.T @ x_deq[:, : ctx.w_k]
            return None, None, dx, None, dw, None
        x_theta, x_q, x_alpha, w_theta, w_q, w_alpha = ctx.saved_tensors
        deq = _DEQ[ctx.fmt]
        dx = dw = None
        if ctx.fmt == "mxfp8":
            x_theta = x_theta.view(torch.float8_e4m3fn)
            w_theta = w_theta.view(torch.float8_e4m3fn)
        if ctx.x_k is not None:
            dx = grad_output @ deq(w_theta, w_q, w_alpha)[:, : ctx.x_k]
        if ctx.w_k is not None:
            dw = grad_output.T @ _dequant_activation(deq, x_theta, x_q, x_alpha, {})[:, : ctx.w_k]
        return None, None, dx, None, dw, None


def make_matmul(fmt: str, quantized_backward: bool = False):
    def matmul(x: QTensor, w: QTensor) -> torch.Tensor:
        return BlockScaledMatMul.apply(fmt, x, x.proxy(), w, w.proxy(), quantized_backward)

    return matmul
