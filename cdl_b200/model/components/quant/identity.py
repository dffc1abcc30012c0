"""No-op quantizer, mirroring ``cdl.model.components.quant.identity``
(cdl/model/components/quant/identity.py): the tensor passes unchanged and
has no gradient proxy."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from cdl_b200.api.quant import QTensor, Quant


@dataclass
class IdentityTensor(QTensor):
    theta: torch.Tensor

    def dequantize(self) -> torch.Tensor:
        return self.theta

    def proxy(self) -> torch.Tensor | None:
        return None


class IdentityQuant(Quant):
    def forward(self, x: torch.Tensor) -> IdentityTensor:
        return IdentityTensor(theta=x)
