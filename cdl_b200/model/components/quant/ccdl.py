"""CCDL quantizer modules: the kernel path of
``cdl.model.components.quant.ccdl`` (ccdl.py:67-393 ``CascadedCdlQuant``,
its activation / weight subclasses and mixin; nvfp4.py / mxfp4.py /
mxfp8.py).

A CCDL quantizer learns its block scales: ``log_q`` (one per block of the
declared input shape; a leading dimension declared as 1 shares its scales),
``log_alpha`` (a tensor-wide factor) and two temperatures, ``log_theta_kappa``
and ``log_q_kappa``.  In training mode the forward samples the scales and
the codes with the CCDL kernels (``cdl_b200.core.kernel.ccdl``) and returns
a packed QTensor whose ``proxy()`` carries the CDL proxy gradient back to the
input, q, alpha and both kappas; in eval mode it rounds to the nearest
scale and code (``ccdl_round``, cdl's ``cascaded_nearest_round``).

cdl's modules take ``kernel="torch"`` (a torch sampler with torch's random
stream) or ``"triton"`` (the fused kernels); both names are accepted here and
both run the B200 kernels, whose stream is the Triton kernel's.
"""

from __future__ import annotations

import math
from collections.abc import Iterable
from dataclasses import dataclass
from typing import Literal

import torch
from torch import nn

from cdl_b200.api.quant import QTensor, Quant
from cdl_b200.core.kernel.ccdl import ccdl_quant, ccdl_round
from cdl_b200.core.kernel.dequant import mxfp4_dequant, mxfp8_dequant, nvfp4_dequant
from cdl_b200.core.kernel.ecdl import FormatId
from cdl_b200.model.components.quant.ecdl import group_tensor_into_blocks

Kernel = Literal["torch", "triton"]


@dataclass(frozen=True)
class _Spec:
    block: int
    fid: FormatId
    theta_n: int  # theta levels
    theta_bits: int  # cdl's Format.bits: (n - 1).bit_length()
    q_n: int  # scale levels
    q_max_theta: float  # largest theta level (init_q_from_block_amax divides by it)
    dequant: object


_SPECS = {
    "nvfp4": _Spec(16, FormatId.NVFP4, 16, 4, 126, 6.0, nvfp4_dequant),
    "mxfp4": _Spec(32, FormatId.MXFP4, 16, 4, 255, 6.0, mxfp4_dequant),
    "mxfp8": _Spec(32, FormatId.MXFP8, 254, 8, 255, 448.0, mxfp8_dequant),
}


@dataclass
class PackedCcdlTensor(QTensor):
    """Codes ``[..., nb, cols]``, scale bytes (``[..., nb, 1]``, or q's shape
    when the scales are shared) and alpha of a CCDL quantize: cdl's
    ``Packed{Nvfp4,Mxfp4,Mxfp8}CascadedCdlTensor`` (training) and, with
    ``eval_dtype`` set, its ``{Nvfp4,...}CascadedCdlTensor`` (eval), whose
    ``dequantize`` is ``level * q_level * alpha`` in the level dtype (with
    fp32 levels the dequantize kernel still rounds the product to bf16)."""

    fmt: str
    packed_theta: torch.Tensor
    packed_scale: torch.Tensor
    alpha: torch.Tensor
    grad_proxy: torch.Tensor | None
    k_dim: int
    dtype: torch.dtype
    eval_dtype: torch.dtype | None = None

    def _encoding(self, fmt: str):
        if fmt != self.fmt:
            raise NotImplementedError(f"{self.fmt} tensor has no {fmt} encoding")
        return self.packed_theta.flatten(-2), self.packed_scale.flatten(-2), self.alpha.float().reshape(1)

    def nvfp4(self):
        return self._encoding("nvfp4")

    def mxfp4(self):
        return self._encoding("mxfp4")

    def mxfp8(self):
        return self._encoding("mxfp8")

    def dequantize(self) -> torch.Tensor:
        packed, scale, alpha = self._encoding(self.fmt)
        lead = packed.shape[:-1]
        packed = packed.reshape(-1, packed.shape[-1])
        scale = scale.reshape(-1, scale.shape[-1])
        if scale.shape[0] != packed.shape[0]:
            scale = scale.expand(packed.shape[0], -1)
        if self.eval_dtype is not None:
            # (level * q_level) is exact; alpha enters rounded to the level
            # dtype, as ``alpha.to(theta.dtype)`` in cdl (ccdl.py:43-48)
            alpha = alpha.to(self.eval_dtype).float()
        out = _SPECS[self.fmt].dequant(packed, scale, alpha)
        out = out.reshape(*lead, -1)[..., : self.k_dim]
        return out.to(self.eval_dtype if self.eval_dtype is not None else self.dtype)

    def proxy(self) -> torch.Tensor | None:
        if self.grad_proxy is None:
            return None
        return self.grad_proxy.flatten(-2)[..., : self.k_dim]


@dataclass
class CascadedCdlBypassTensor(QTensor):
    theta: torch.Tensor

    def dequantize(self) -> torch.Tensor:
        return self.theta

    def proxy(self) -> torch.Tensor | None:
        return None


class CascadedCdlQuant(Quant):
    """One CCDL quantizer (ccdl.py:67-207)."""

    def __init__(self, fmt: str, input_shape: tuple[int, ...], theta_topk: int, q_topk: int, dtype: torch.dtype,
                 kappa: float, kernel: Kernel = "triton"):
        super().__init__()
        if fmt not in _SPECS:
            raise ValueError(f"unknown format {fmt!r}")
        if kernel not in ("torch", "triton"):
            raise ValueError(f"unknown kernel {kernel!r}")
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"level dtype must be bf16 or fp32, got {dtype}")
        spec = _SPECS[fmt]
        if not 1 <= theta_topk <= spec.theta_n:
            raise ValueError(f"theta_topk {theta_topk} out of range")
        if not 1 <= q_topk <= spec.q_n:
            raise ValueError(f"q_topk {q_topk} out of range")
        self.fmt, self.spec, self.kernel, self.dtype = fmt, spec, kernel, dtype
        self.block_size, self.theta_topk, self.q_topk = spec.block, theta_topk, q_topk
        self.input_shape = tuple(input_shape)
        self.k_dim = self.input_shape[-1]
        num_blocks = (self.k_dim + spec.block - 1) // spec.block
        self.q_num_quantized_params = math.prod(self.input_shape[:-1]) * num_blocks
        self.theta_num_quantized_params = math.prod(self.input_shape[:-1]) * self.k_dim
        q_shape = self.input_shape[:-1] + (num_blocks, 1)
        self.log_theta_kappa = nn.Parameter(torch.full((), math.log(kappa)))
        self.log_q_kappa = nn.Parameter(torch.full((), math.log(kappa)))
        self.log_q = nn.Parameter(torch.zeros(q_shape))
        self.log_alpha = nn.Parameter(torch.zeros(()))
        self.register_buffer("log_q_init", self.log_q.detach().clone(), persistent=False)
        self.register_buffer("kernel_seed", torch.zeros((), dtype=torch.int64), persistent=False)
        self.initialized = False
        self.bypassing = False

    @property
    def theta_kappa(self) -> torch.Tensor:
        return self.log_theta_kappa.exp()

    @property
    def q_kappa(self) -> torch.Tensor:
        return self.log_q_kappa.exp()

    @property
    def q(self) -> torch.Tensor:
        return self.log_q.exp()

    @property
    def alpha(self) -> torch.Tensor:
        return self.log_alpha.exp()

    # learning rates (ccdl.py:124-134, 231-240, 264-273)
    def _lr_bits(self) -> int:
        return self.spec.theta_bits

    def get_q_lr(self, eta: float) -> float:
        return eta / math.sqrt(self.block_size * (2 ** self._lr_bits()))

    def get_alpha_lr(self, eta: float) -> float:
        return eta / math.sqrt(self.theta_num_quantized_params * (2 ** self._lr_bits()))

    def get_theta_kappa_lr(self, eta: float) -> float:
        return eta / self.theta_num_quantized_params ** 0.5

    def get_q_kappa_lr(self, eta: float) -> float:
        return eta / self.log_q.numel() ** 0.5

    @torch.no_grad()
    def copy_log_q(self, log_q_tensor: torch.Tensor) -> None:
        self.log_q.copy_(log_q_tensor)
        self.log_q_init.copy_(log_q_tensor)

    @torch.no_grad()
    def init_q_from_block_amax(self, block_amax: torch.Tensor) -> None:
        """q = block amax / largest theta level, floored at the smallest
        normal fp32, logarithm in the amax dtype (ccdl.py:141-144)."""
        top = torch.tensor(self.spec.q_max_theta, dtype=self.dtype, device=block_amax.device)
        q = block_amax / top
        self.copy_log_q(q.clamp_min(torch.finfo(torch.float32).tiny).log())

    def eval_forward(self, theta: torch.Tensor) -> QTensor:
        packed, scale = ccdl_round(theta, self.q.detach(), self.alpha.detach(), self.spec.fid, self.dtype)
        return PackedCcdlTensor(self.fmt, packed, scale, self.alpha.detach(), None, self.k_dim, self.dtype,
                                eval_dtype=self.dtype)

    def training_forward(self, theta: torch.Tensor) -> QTensor:
        packed, scale, carrier = ccdl_quant(theta, self.q, self.theta_kappa, self.q_kappa, self.alpha,
                                            self.kernel_seed, self.spec.fid, self.theta_topk, self.q_topk)
        return PackedCcdlTensor(self.fmt, packed, scale, self.alpha.detach(), carrier, self.k_dim, self.dtype)

    def forward(self, x: torch.Tensor) -> QTensor:
        if self.bypassing:
            return CascadedCdlBypassTensor(x)
        if not self.initialized:
            raise RuntimeError("CCDL quantizer used before its scales were initialized")
        if x.ndim != len(self.input_shape) or any(d != 1 and d != a for d, a in zip(self.input_shape, x.shape)):
            raise ValueError(f"expected input shaped like {self.input_shape}, got {tuple(x.shape)}")
        theta, _ = group_tensor_into_blocks(x, self.block_size)
        return self.training_forward(theta) if self.training else self.eval_forward(theta)


class CascadedCdlQuantForActivation(CascadedCdlQuant):
    """Activation quantizer: scales from a calibration pass
    (``CascadedCdlQuantMixin.cascaded_cdl_init_act_q_pass``)."""

    FMT = ""

    def __init__(self, input_shape: tuple[int, ...], theta_topk: int, q_topk: int, dtype: torch.dtype, kappa: float,
                 kernel: Kernel = "torch"):
        super().__init__(self.FMT, input_shape, theta_topk, q_topk, dtype, kappa, kernel)


class CascadedCdlQuantForWeight(CascadedCdlQuant):
    """Weight quantizer: samples from the whole grids, scales from the
    weight's block amax (ccdl.py:242-278)."""

    FMT = ""

    def __init__(self, weight: torch.Tensor, dtype: torch.dtype, kappa: float, kernel: Kernel = "torch"):
        spec = _SPECS[self.FMT]
        super().__init__(self.FMT, tuple(weight.shape), spec.theta_n, spec.q_n, dtype, kappa, kernel)
        self.init_q_from_weight(weight)
        self.initialized = True

    def _lr_bits(self) -> int:
        return self.spec.theta_bits - 1

    @torch.no_grad()
    def init_q_from_weight(self, weight: torch.Tensor) -> None:
        blocked, _ = group_tensor_into_blocks(weight, self.block_size)
        self.init_q_from_block_amax(blocked.abs().amax(dim=-1, keepdim=True))


class Nvfp4CascadedCdlQuantForActivation(CascadedCdlQuantForActivation):
    FMT = "nvfp4"


class Nvfp4CascadedCdlQuantForWeight(CascadedCdlQuantForWeight):
    FMT = "nvfp4"


class Mxfp4CascadedCdlQuantForActivation(CascadedCdlQuantForActivation):
    FMT = "mxfp4"


class Mxfp4CascadedCdlQuantForWeight(CascadedCdlQuantForWeight):
    FMT = "mxfp4"


class Mxfp8CascadedCdlQuantForActivation(CascadedCdlQuantForActivation):
    FMT = "mxfp8"


class Mxfp8CascadedCdlQuantForWeight(CascadedCdlQuantForWeight):
    FMT = "mxfp8"


class CascadedCdlQuantMixin(nn.Module):
    """Model-level helpers of cdl's ``CascadedCdlQuantMixin`` (ccdl.py:280-393):
    quantized-element counts, statistics, optimizer parameter groups and the
    activation-scale calibration pass.  (cdl's mixin also puts BatchNorm2d
    layers in batch-statistics mode during calibration; the decoder models
    here have none.)"""

    def cascaded_cdl_get_weight_quant_counts(self) -> int:
        return sum(m.theta_num_quantized_params for m in self.modules() if isinstance(m, CascadedCdlQuantForWeight))

    def cascaded_cdl_get_activation_quant_counts(self) -> int:
        return sum(m.theta_num_quantized_params for m in self.modules()
                   if isinstance(m, CascadedCdlQuantForActivation))

    @torch.no_grad()
    def cascaded_cdl_quant_stats(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for name, m in self.named_modules():
            if not isinstance(m, CascadedCdlQuant):
                continue
            name = name.removeprefix("_orig_mod.")
            out[f"{name}.theta_kappa"] = m.theta_kappa.item()
            out[f"{name}.q"] = m.q.detach().float().mean().item()
            out[f"{name}.q_rel"] = (m.log_q - m.log_q_init).float().abs().mean().item()
            out[f"{name}.q_kappa"] = m.q_kappa.item()
            out[f"{name}.alpha"] = m.alpha.item()
        return out

    @torch.no_grad()
    def cascaded_cdl_get_param_groups(self, learning_rate: float, train_alpha: bool,
                                      train_kappa: bool) -> tuple[list[dict], set[nn.Parameter]]:
        custom: set[nn.Parameter] = set()
        buckets: dict[float, list[nn.Parameter]] = {}
        for m in self.modules():
            if not isinstance(m, CascadedCdlQuant):
                continue
            custom.update(m.parameters())
            buckets.setdefault(m.get_q_lr(learning_rate), []).append(m.log_q)
            if train_alpha:
                buckets.setdefault(m.get_alpha_lr(learning_rate), []).append(m.log_alpha)
            else:
                m.log_alpha.requires_grad_(False)
            if train_kappa:
                buckets.setdefault(m.get_theta_kappa_lr(learning_rate), []).append(m.log_theta_kappa)
                buckets.setdefault(m.get_q_kappa_lr(learning_rate), []).append(m.log_q_kappa)
            else:
                m.log_theta_kappa.requires_grad_(False)
                m.log_q_kappa.requires_grad_(False)
        groups = [{"params": params, "lr": lr, "weight_decay": 0.0} for lr, params in buckets.items()]
        return groups, custom

    @torch.no_grad()
    def cascaded_cdl_init_act_q_pass(self, samples: Iterable[torch.Tensor]) -> None:
        """Runs the model in eval mode with the activation quantizers bypassed,
        records each one's block amax (max over the batch-like dimensions its
        input shape declares as 1, and over the samples) and sets q from it."""
        modules = [m for m in self.modules() if isinstance(m, CascadedCdlQuantForActivation)]
        if not modules:
            return
        stats: dict[CascadedCdlQuantForActivation, torch.Tensor] = {}

        def hook(m, args):
            blocked, _ = group_tensor_into_blocks(args[0], m.block_size)
            dims = tuple(i for i in range(blocked.ndim - 2) if m.input_shape[i] == 1) + (blocked.ndim - 1,)
            amax = blocked.abs().amax(dim=dims)
            prev = stats.get(m)
            stats[m] = amax if prev is None else torch.maximum(prev, amax)

        handles = [m.register_forward_pre_hook(hook) for m in modules]
        was_training = self.training
        self.eval()
        for m in modules:
            m.bypassing = True
        try:
            for x in samples:
                self(x)
        finally:
            for h in handles:
                h.remove()
            for m in modules:
                m.bypassing = False
            self.train(was_training)
        for m in modules:
            if m not in stats:
                raise RuntimeError("an activation quantizer saw no calibration input")
            m.init_q_from_block_amax(stats[m].flatten().reshape(m.input_shape[:-1] + (-1, 1)))
            m.initialized = True
