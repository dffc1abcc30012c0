"""Quantized linear layer, mirroring ``cdl.model.components.linear``
(cdl/model/components/linear.py:14-103).

``QLinear`` quantizes its activation and (LoRA-merged) weight through its
``Quant`` modules and multiplies them with the matmul backend named by
``backend``: ``native`` (dequantize, then bf16 matmul), ``nvfp4`` / ``mxfp4``
/ ``mxfp8`` (B200 block-scaled GEMM forward, bf16 backward as cdl), and
``nvfp4_qbwd`` / ``mxfp4_qbwd`` / ``mxfp8_qbwd`` (dgrad and wgrad in the same
block-scaled format too).
"""

from __future__ import annotations

import math
from typing import Any, Literal

import torch
from torch import nn

from cdl_b200.api.quant import MatMul, Quant
from cdl_b200.core.mm import mxfp4, mxfp8, native, nvfp4
from cdl_b200.model.components.quant.ste import SteQuant

Backend = Literal["native", "nvfp4", "mxfp4", "mxfp8", "nvfp4_qbwd", "mxfp4_qbwd", "mxfp8_qbwd"]


class MergedLoRALayer(nn.Module):
    def __init__(self, hint: nn.Linear, r: int, alpha: int) -> None:
        super().__init__()
        device, dtype = hint.weight.device, hint.weight.dtype
        self.r = r
        self.scaling = alpha / r
        self.a = nn.Parameter(torch.empty(r, hint.in_features, device=device, dtype=dtype))
        nn.init.kaiming_uniform_(self.a, a=math.sqrt(5))
        self.b = nn.Parameter(torch.zeros(hint.out_features, r, device=device, dtype=dtype))

    def forward(self, weight: torch.Tensor) -> torch.Tensor:
        return weight + self.scaling * (self.b @ self.a)


_BACKENDS: dict[str, MatMul] = {
    "native": native.matmul,
    "nvfp4": nvfp4.matmul,
    "mxfp4": mxfp4.matmul,
    "mxfp8": mxfp8.matmul,
    "nvfp4_qbwd": nvfp4.matmul_qbwd,
    "mxfp4_qbwd": mxfp4.matmul_qbwd,
    "mxfp8_qbwd": mxfp8.matmul_qbwd,
}


class QLinear(nn.Linear):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device: Any | None = None,
                 dtype: Any | None = None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self.activation_quant: Quant = SteQuant(None)
        self.weight_quant: Quant = SteQuant(None)
        self.backend = "native"
        self.lora: nn.Module = nn.Identity()

    def set_activation_quant(self, quant: Quant) -> None:
        self.activation_quant = quant

    def set_weight_quant(self, quant: Quant) -> None:
        self.weight_quant = quant

    def set_backend(self, backend: Backend) -> None:
        if backend not in _BACKENDS:
            raise ValueError(f"unknown backend {backend!r}")
        self.backend = backend

    def set_lora(self, r: int, alpha: int) -> None:
        self.lora = MergedLoRALayer(self, r, alpha)

    @property
    def available_backend_fn(self) -> dict[str, MatMul]:
        return dict(_BACKENDS)

    @staticmethod
    def from_linear(linear: nn.Linear) -> "QLinear":
        new = QLinear(linear.in_features, linear.out_features, bias=linear.bias is not None,
                      device=linear.weight.device, dtype=linear.weight.dtype)
        with torch.no_grad():
            new.weight.copy_(linear.weight)
            if linear.bias is not None:
                new.bias.copy_(linear.bias)
        new.weight.requires_grad_(linear.weight.requires_grad)
        if linear.bias is not None:
            new.bias.requires_grad_(linear.bias.requires_grad)
        return new

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2d = x.reshape(-1, x.shape[-1])
        activation = self.activation_quant(x2d)
        weight = self.weight_quant(self.lora(self.weight))
        out = _BACKENDS[self.backend](activation, weight)
        if self.bias is not None:
            out = out + self.bias
        return out.reshape(*x.shape[:-1], -1)


class QLinearMixin(nn.Module):
    def q_linear_switch_backend(self, backend: Backend) -> None:
        for m in self.modules():
            if isinstance(m, QLinear):
                m.set_backend(backend)
