"""Dequantize-then-matmul backend with the STE, mirroring
``cdl.core.mm.native`` (cdl/core/mm/native.py:6-17): ``proxy + (deq - proxy)
.detach()`` for each operand, then a bf16 matmul."""

from __future__ import annotations

import torch

from cdl_b200.api.quant import QTensor


def matmul(x: QTensor, w: QTensor) -> torch.Tensor:
    fp_x = x.dequantize()
    fp_x_proxy = x.proxy()
    if fp_x_proxy is not None:
        fp_x = fp_x_proxy + (fp_x - fp_x_proxy).detach()
    fp_w = w.dequantize()
    fp_w_proxy = w.proxy()
    if fp_w_proxy is not None:
        fp_w = fp_w_proxy + (fp_w - fp_w_proxy).detach()
    return fp_x @ fp_w.T
