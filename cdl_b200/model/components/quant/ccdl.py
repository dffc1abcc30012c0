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
from cdl_b200.model.components.quant.identity import IdentityTensor

Kernel = Literal["torch", "triton"]


def _unblock(t: torch.Tensor, k: int) -> torch.Tensor:
    """``[..., nb, block]`` back to ``[..., k]`` (the padded tail dropped)."""
    return t.flatten(-2)[..., :k]


def _block_amax(t: torch.Tensor, block: int) -> torch.Tensor:
    """max |t| of each block of ``block`` along the last dim, ``[..., nb, 1]``."""
    blocked, _ = group_tensor_into_blocks(t, block)
    return blocked.abs().amax(dim=-1, keepdim=True)


class _Exp:
    """Read-only attribute ``exp(<name>)`` of a log-parameterised parameter."""

    def __init__(self, name: str):
        self.name = name

    def __get__(self, obj, owner=None):
        return self if obj is None else getattr(obj, self.name).exp()


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
        return None if self.grad_proxy is None else _unblock(self.grad_proxy, self.k_dim)


class CascadedCdlBypassTensor(IdentityTensor):
    """What a bypassing quantizer (activation calibration) returns: the input
    itself, no gradient proxy -- cdl's ``CascadedCdlBypassTensor``."""


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

    # the learned quantities, stored as logarithms
    theta_kappa = _Exp("log_theta_kappa")
    q_kappa = _Exp("log_q_kappa")
    q = _Exp("log_q")
    alpha = _Exp("log_alpha")

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
        """Set log q and remember it as the starting point of ``q_rel``."""
        for dst in (self.log_q, self.log_q_init):
            dst.copy_(log_q_tensor)

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
        """q from the weight's own block maxima (cdl: ccdl.py:273-279)."""
        self.init_q_from_block_amax(_block_amax(weight, self.block_size))


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


# per-quantizer statistics of cdl's ``cascaded_cdl_quant_stats``
# (ccdl.py:294-310): name suffix -> value
_STATS = {
    "theta_kappa": lambda m: m.theta_kappa,
    "q": lambda m: m.q.detach().float().mean(),
    "q_rel": lambda m: (m.log_q - m.log_q_init).float().abs().mean(),
    "q_kappa": lambda m: m.q_kappa,
    "alpha": lambda m: m.alpha,
}


class _AmaxRecorder:
    """Calibration context: the activation quantizers pass their input through
    (``bypassing``), the model runs in eval mode, and a forward pre-hook keeps
    the running block amax of each quantizer's input, reduced over the
    dimensions its declared input shape marks as 1 (shared scales)."""

    def __init__(self, model: nn.Module, quantizers: list):
        self.model, self.quantizers = model, quantizers
        self.amax: dict = {}
        self._handles: list = []
        self._was_training = model.training

    def _hook(self, m, args):
        blocked, _ = group_tensor_into_blocks(args[0], m.block_size)
        shared = [i for i in range(blocked.ndim - 2) if m.input_shape[i] == 1]
        seen = blocked.abs().amax(dim=(*shared, blocked.ndim - 1))
        old = self.amax.get(m)
        self.amax[m] = seen if old is None else torch.maximum(old, seen)

    def __enter__(self):
        self._handles = [m.register_forward_pre_hook(self._hook) for m in self.quantizers]
        self.model.eval()
        for m in self.quantizers:
            m.bypassing = True
        return self

    def __exit__(self, *exc):
        for h in self._handles:
            h.remove()
        for m in self.quantizers:
            m.bypassing = False
        self.model.train(self._was_training)
        return False


class CascadedCdlQuantMixin(nn.Module):
    """Model-level helpers of cdl's ``CascadedCdlQuantMixin`` (ccdl.py:280-393):
    quantized-element counts, statistics, optimizer parameter groups and the
    activation-scale calibration pass.  (cdl's mixin also puts BatchNorm2d
    layers in batch-statistics mode during calibration; the decoder models
    here have none.)"""

    def _ccdl_quantizers(self, kind=None) -> list:
        kind = kind or CascadedCdlQuant
        return [m for m in self.modules() if isinstance(m, kind)]

    def cascaded_cdl_get_weight_quant_counts(self) -> int:
        return sum(m.theta_num_quantized_params for m in CascadedCdlQuantMixin._ccdl_quantizers(
            self, CascadedCdlQuantForWeight))

    def cascaded_cdl_get_activation_quant_counts(self) -> int:
        return sum(m.theta_num_quantized_params for m in CascadedCdlQuantMixin._ccdl_quantizers(
            self, CascadedCdlQuantForActivation))

    @torch.no_grad()
    def cascaded_cdl_quant_stats(self) -> dict[str, float]:
        """``<module name>.<stat>`` for every quantizer and statistic in _STATS
        (names without a torch.compile ``_orig_mod.`` prefix)."""
        return {f"{name.removeprefix('_orig_mod.')}.{stat}": float(fn(m))
                for name, m in self.named_modules() if isinstance(m, CascadedCdlQuant)
                for stat, fn in _STATS.items()}

    @torch.no_grad()
    def cascaded_cdl_get_param_groups(self, learning_rate: float, train_alpha: bool,
                                      train_kappa: bool) -> tuple[list[dict], set[nn.Parameter]]:
        """One AdamW group per distinct learning rate: log q always, log alpha
        and the two log kappas when trained (else frozen); returns the groups
        and the set of every quantizer parameter."""
        owned: set[nn.Parameter] = set()
        by_lr: dict[float, list[nn.Parameter]] = {}
        for m in CascadedCdlQuantMixin._ccdl_quantizers(self):
            owned.update(m.parameters())
            entries = [(m.log_q, m.get_q_lr, True), (m.log_alpha, m.get_alpha_lr, train_alpha),
                       (m.log_theta_kappa, m.get_theta_kappa_lr, train_kappa),
                       (m.log_q_kappa, m.get_q_kappa_lr, train_kappa)]
            for param, lr_of, trained in entries:
                if trained:
                    by_lr.setdefault(lr_of(learning_rate), []).append(param)
                else:
                    param.requires_grad_(False)
        return [{"params": ps, "lr": lr, "weight_decay": 0.0} for lr, ps in by_lr.items()], owned

    @torch.no_grad()
    def cascaded_cdl_init_act_q_pass(self, samples: Iterable[torch.Tensor]) -> None:
        """Calibrate every activation quantizer's q from the block amax of its
        input over ``samples`` (cdl: ccdl.py:356-393)."""
        quantizers = CascadedCdlQuantMixin._ccdl_quantizers(self, CascadedCdlQuantForActivation)
        if not quantizers:
            return
        with _AmaxRecorder(self, quantizers) as rec:
            for x in samples:
                self(x)
        for m in quantizers:
            if m not in rec.amax:
                raise RuntimeError("an activation quantizer saw no calibration input")
            m.init_q_from_block_amax(rec.amax[m].flatten().reshape(m.input_shape[:-1] + (-1, 1)))
            m.initialized = True
