"""Quantizer interfaces, mirroring ``cdl.api.quant`` (cdl/api/quant.py:8-30).

A :class:`QTensor` hands its block-scaled encodings to a matmul backend
(``nvfp4()`` / ``mxfp4()`` / ``mxfp8()`` -> ``(codes, scales, alpha)``), can
``dequantize()`` itself, and exposes the tensor gradients flow to
(``proxy()``).  A :class:`Quant` module turns a tensor into a QTensor; a
``MatMul`` is any ``(QTensor, QTensor) -> Tensor`` callable.
"""

from __future__ import annotations

import abc
from collections.abc import Callable

import torch
from torch import nn


class QTensor(abc.ABC):
    def nvfp4(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        raise NotImplementedError()

    def mxfp4(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        raise NotImplementedError()

    def mxfp8(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
        raise NotImplementedError()

    @abc.abstractmethod
    def dequantize(self) -> torch.Tensor: ...

    def proxy(self) -> torch.Tensor | None:
        raise NotImplementedError()


class Quant(nn.Module, abc.ABC):
    @abc.abstractmethod
    def forward(self, x: torch.Tensor) -> QTensor: ...


MatMul = Callable[[QTensor, QTensor], torch.Tensor]
