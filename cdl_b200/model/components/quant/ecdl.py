"""ECDL quantizer modules: the kernel path of
``cdl.model.components.quant.ecdl`` (ecdl.py:16-196 ``ExtendedCdlQuant`` and
its activation / weight subclasses, nvfp4.py / mxfp4.py / mxfp8.py).

In training mode a module samples its input's codes with the ECDL kernels
(``cdl_b200.core.kernel.ecdl``) and returns a packed QTensor whose
``proxy()`` carries the CDL proxy gradient back to the input and to
``log_kappa``; in eval mode it rounds deterministically (the block-scaled
quantizers).  The QTensor feeds any matmul backend through ``nvfp4()`` /
``mxfp4()`` / ``mxfp8()``.

cdl's modules take ``kernel="torch"`` (a pure-torch sampler with torch's
random stream) or ``"triton"`` (the fused kernels); both names are accepted
here and both run the B200 kernels, whose stream is the Triton kernel's.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import nn

from cdl_b200.api.quant import QTensor, Quant
from cdl_b200.core.kernel.dequant import mxfp4_dequant, mxfp8_dequant, nvfp4_dequant
from cdl_b200.core.kernel.ecdl import FormatId, ecdl_quant
from cdl_b200.core.kernel.quant import mxfp4_quant, mxfp8_quant, nvfp4_quant

Kernel = Literal["torch", "triton"]

# format -> (block, format id, scale mode, theta levels, deterministic quantizer, dequantizer)
_FORMATS = {
    "nvfp4": (16, FormatId.NVFP4, "nvidia", 16, nvfp4_quant, nvfp4_dequant),
    "mxfp4": (32, FormatId.MXFP4, "ocp", 16, mxfp4_quant, mxfp4_dequant),
    "mxfp8": (32, FormatId.MXFP8, "ocp", 254, mxfp8_quant, mxfp8_dequant),
}


def group_tensor_into_blocks(theta: torch.Tensor, block_size: int) -> tuple[torch.Tensor, int]:
    """``[..., K]`` -> ``[..., nb, block]``, zero-padding K (ecdl.py:16-29)."""
    k = theta.shape[-1]
    pad = (-k) % block_size
    if pad:
        theta = F.pad(theta, (0, pad))
    return theta.reshape(*theta.shape[:-1], (k + pad) // block_size, block_size), pad


@dataclass
class PackedEcdlTensor(QTensor):
    """Codes ``[..., nb, cols]``, scale bytes ``[..., nb, 1]`` and alpha of an
    ECDL (or eval-mode) quantize; cdl's ``Packed*ExtendedCdlTensor``."""

    fmt: str
    packed_theta: torch.Tensor
    packed_scale: torch.Tensor
    alpha: torch.Tensor | None
    grad_proxy: torch.Tensor | None
    k_dim: int
    dtype: torch.dtype

    def _encoding(self, fmt: str):
        if fmt != self.fmt:
            raise NotImplementedError(f"{self.fmt} tensor has no {fmt} encoding")
        alpha = None if self.alpha is None or fmt == "mxfp8" else self.alpha.float().reshape(1)
        return self.packed_theta.flatten(-2), self.packed_scale.flatten(-2), alpha

    def nvfp4(self):
        return self._encoding("nvfp4")

    def mxfp4(self):
        return self._encoding("mxfp4")

    def mxfp8(self):
        return self._encoding("mxfp8")

    def dequantize(self) -> torch.Tensor:
        packed, scale, alpha = self._encoding(self.fmt)
        lead = packed.shape[:-1]
        deq = _FORMATS[self.fmt][5]
        if self.fmt == "mxfp8":
            out = deq(packed.reshape(-1, packed.shape[-1]), scale.reshape(-1, scale.shape[-1]), None)
        else:
            a = alpha if alpha is not None else torch.ones(1, device=packed.device)
            out = deq(packed.reshape(-1, packed.shape[-1]), scale.reshape(-1, scale.shape[-1]), a)
        return out.reshape(*lead, -1)[..., : self.k_dim].to(self.dtype)

    def proxy(self) -> torch.Tensor | None:
        if self.grad_proxy is None:
            return None
        return self.grad_proxy.flatten(-2)[..., : self.k_dim]


@dataclass
class EcdlBypassTensor(QTensor):
    theta: torch.Tensor

    def dequantize(self) -> torch.Tensor:
        return self.theta

    def proxy(self) -> torch.Tensor | None:
        return None


class ExtendedCdlQuant(Quant):
    """One ECDL quantizer: learnable ``log_kappa`` (forward temperature), an
    optional fixed backward ``kappa_backward``, the kernel seed (advanced by
    every training forward)."""

    def __init__(self, fmt: str, input_shape: tuple[int, ...], theta_topk: int, dtype: torch.dtype,
                 kappa_forward: float, kappa_backward: float | None = None, kernel: Kernel = "triton"):
        super().__init__()
        if fmt not in _FORMATS:
            raise ValueError(f"unknown format {fmt!r}")
        if kernel not in ("torch", "triton"):
            raise ValueError(f"unknown kernel {kernel!r}")
        block, _, _, tn, _, _ = _FORMATS[fmt]
        if not 1 <= theta_topk <= tn:
            raise ValueError(f"theta_topk {theta_topk} out of range")
        self.fmt, self.block_size, self.theta_topk, self.dtype, self.kernel = fmt, block, theta_topk, dtype, kernel
        self.input_shape = tuple(input_shape)
        self.k_dim = self.input_shape[-1]
        self.num_quantized_params = math.prod(self.input_shape)
        self.log_kappa = nn.Parameter(torch.full((), math.log(kappa_forward)))
        if kappa_backward is not None:
            self.register_buffer("kappa_backward", torch.tensor(kappa_backward, dtype=torch.float32),
                                 persistent=False)
        else:
            self.register_buffer("kappa_backward", None, persistent=False)
        self.register_buffer("kernel_seed", torch.zeros((), dtype=torch.int64), persistent=False)
        self.bypassing = False

    @property
    def kappa(self) -> torch.Tensor:
        return self.log_kappa.exp()

    def eval_forward(self, theta: torch.Tensor) -> QTensor:
        lead, (nb, tpb) = theta.shape[:-2], theta.shape[-2:]
        packed, scale, alpha = _FORMATS[self.fmt][4](theta.reshape(-1, nb * tpb))
        return PackedEcdlTensor(self.fmt, packed.reshape(*lead, nb, packed.shape[-1] // nb),
                                scale.reshape(*lead, nb, 1), None if alpha is None else alpha.detach(), None,
                                self.k_dim, self.dtype)

    def training_forward(self, theta: torch.Tensor) -> QTensor:
        _, fid, mode, _, _, _ = _FORMATS[self.fmt]
        packed, scale, carrier, alpha = ecdl_quant(theta, self.kappa, self.kappa_backward, self.kernel_seed, fid,
                                                   self.theta_topk, mode)
        return PackedEcdlTensor(self.fmt, packed, scale, None if self.fmt == "mxfp8" else alpha.detach(), carrier,
                                self.k_dim, self.dtype)

    def forward(self, x: torch.Tensor) -> QTensor:
        if self.bypassing:
            return EcdlBypassTensor(x)
        if x.ndim != len(self.input_shape) or any(d != 1 and d != a for d, a in zip(self.input_shape, x.shape)):
            raise ValueError(f"expected input shaped like {self.input_shape}, got {tuple(x.shape)}")
        theta, _ = group_tensor_into_blocks(x, self.block_size)
        return self.training_forward(theta) if self.training else self.eval_forward(theta)


class _ForActivation(ExtendedCdlQuant):
    FMT = ""

    def __init__(self, input_shape: tuple[int, ...], theta_topk: int, dtype: torch.dtype, kappa_forward: float,
                 kappa_backward: float | None = None, kernel: Kernel = "torch"):
        super().__init__(self.FMT, input_shape, theta_topk, dtype, kappa_forward, kappa_backward, kernel)


class _ForWeight(ExtendedCdlQuant):
    FMT = ""

    def __init__(self, weight: torch.Tensor, dtype: torch.dtype, kappa_forward: float, kernel: Kernel = "torch"):
        # weights sample from the whole level grid (ecdl.py:186-196)
        super().__init__(self.FMT, tuple(weight.shape), _FORMATS[self.FMT][3], dtype, kappa_forward, None, kernel)


class Nvfp4ExtendedCdlQuantForActivation(_ForActivation):
    FMT = "nvfp4"


class Nvfp4ExtendedCdlQuantForWeight(_ForWeight):
    FMT = "nvfp4"


class Mxfp4ExtendedCdlQuantForActivation(_ForActivation):
    FMT = "mxfp4"


class Mxfp4ExtendedCdlQuantForWeight(_ForWeight):
    FMT = "mxfp4"


class Mxfp8ExtendedCdlQuantForActivation(_ForActivation):
    FMT = "mxfp8"


class Mxfp8ExtendedCdlQuantForWeight(_ForWeight):
    FMT = "mxfp8"


class ExtendedCdlQuantMixin(nn.Module):
    """Model-level helpers of cdl's ``ExtendedCdlQuantMixin``
    (ecdl/ecdl.py:213-264): quantized-element counts, kappa statistics and
    the optimizer parameter group of the temperatures."""

    def extended_cdl_get_weight_quant_counts(self) -> int:
        return sum(m.num_quantized_params for m in self.modules() if isinstance(m, _ForWeight))

    def extended_cdl_get_activation_quant_counts(self) -> int:
        return sum(m.num_quantized_params for m in self.modules() if isinstance(m, _ForActivation))

    @torch.no_grad()
    def extended_cdl_quant_stats(self) -> dict[str, float]:
        return {f"{name.removeprefix('_orig_mod.')}.kappa": m.kappa.item()
                for name, m in self.named_modules() if isinstance(m, ExtendedCdlQuant)}

    @torch.no_grad()
    def extended_cdl_get_param_groups(self, learning_rate: float,
                                      train_kappa: bool) -> tuple[list[dict], set[nn.Parameter]]:
        custom: set[nn.Parameter] = set()
        params: list[nn.Parameter] = []
        for m in self.modules():
            if not isinstance(m, ExtendedCdlQuant):
                continue
            custom.update(m.parameters())
            if train_kappa:
                params.append(m.log_kappa)
            else:
                m.log_kappa.requires_grad_(False)
        groups = [{"params": params, "lr": learning_rate, "weight_decay": 0.0}] if params else []
        return groups, custom
