"""Block-scaled matmul with the STE, shared by the ``nvfp4`` / ``mxfp4`` /
``mxfp8`` backends (cdl/core/mm/nvfp4.py:9-63, mxfp4.py:9-63, mxfp8.py:9-70).

Forward: both operands are quantized by the B200 kernels, their scales
swizzled into the 128x4 GEMM layout, and the tcgen05 block-scaled GEMM
produces bf16 ``alpha * deq(x) @ deq(w)^T`` (MXFP8 applies alpha outside the
GEMM, as cdl does).  Backward, as cdl: ``dx = g @ deq(w)``, ``dw = g^T @
deq(x)`` with bf16 operands (the straight-through estimator: gradients flow
to the unquantized proxies).
"""

from __future__ import annotations

import torch

from cdl_b200.api.quant import QTensor
from cdl_b200.core.kernel.dequant import mxfp4_dequant, mxfp8_dequant, nvfp4_dequant
from cdl_b200.core.mm.swizzle import expand_rows, pad_k, pad_n, swizzle_scale_factors
from cdl_b200.model.wrapper.ops import mm_fp4, mm_mxfp8

_DEQ = {"nvfp4": nvfp4_dequant, "mxfp4": mxfp4_dequant, "mxfp8": mxfp8_dequant}


class BlockScaledMatMul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fmt: str, x: QTensor, x_proxy, w: QTensor, w_proxy):
        ctx.fmt = fmt
        ctx.x_k = x_proxy.shape[-1] if x_proxy is not None else None
        ctx.w_k = w_proxy.shape[-1] if w_proxy is not None else None
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
        x_theta, x_q, x_alpha, w_theta, w_q, w_alpha = ctx.saved_tensors
        deq = _DEQ[ctx.fmt]
        dx = dw = None
        if ctx.fmt == "mxfp8":
            x_theta = x_theta.view(torch.float8_e4m3fn)
            w_theta = w_theta.view(torch.float8_e4m3fn)
        if ctx.x_k is not None:
            dx = grad_output @ deq(w_theta, w_q, w_alpha)[:, : ctx.x_k]
        if ctx.w_k is not None:
            dw = grad_output.T @ deq(x_theta, x_q, x_alpha)[:, : ctx.w_k]
        return None, None, dx, None, dw


def make_matmul(fmt: str):
    def matmul(x: QTensor, w: QTensor) -> torch.Tensor:
        return BlockScaledMatMul.apply(fmt, x, x.proxy(), w, w.proxy())

    return matmul
