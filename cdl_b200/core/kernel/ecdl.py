"""ECDL stochastic quantizer: the drop-in for ``cdl.core.kernel.ecdl``
(cdl/core/kernel/ecdl/autograd.py, launch.py) and the format entry points of
``cdl.core.kernel`` (entries.py:79-131).

``ecdl_quant(theta, kappa_forward, kappa_backward, seed, format_id,
theta_topk, scale_mode)`` takes theta grouped into blocks ``[..., nb, tpb]``
(tpb 16 for NVFP4, 32 for MXFP4 / MXFP8) and returns, as the reference does,
``(packed_theta, packed_scale, carrier, alpha_eff)``: the sampled codes, the
scale bytes ``[..., nb, 1]``, a zero tensor shaped like theta whose gradient
is the proxy gradient, and alpha.  The forward increments ``seed`` in place
before sampling.  The backward gives theta the CDL proxy gradient and kappa
(forward kappa when ``kappa_backward`` is None, else the fixed backward one
gets none) its gradient.  Kernels: ``cdlb200_ecdl_fwd`` / ``cdlb200_ecdl_bwd``
(include/cdlb200_step.h); the random stream is Triton's tl.rand (Philox),
so a given seed samples what the reference's kernel samples.
"""

from __future__ import annotations

import math
from enum import IntEnum

import torch

from cdl_b200 import _lib


class FormatId(IntEnum):
    NVFP4 = 0
    MXFP4 = 1
    MXFP8 = 2


_TPB = {FormatId.NVFP4: 16, FormatId.MXFP4: 32, FormatId.MXFP8: 32}
_SCALE_MODES = {"nvidia": 0, "ocp": 1}


def _mode(scale_mode: str) -> int:
    if scale_mode not in _SCALE_MODES:
        raise ValueError(f"unsupported scale mode {scale_mode!r} (nvidia or ocp)")
    return _SCALE_MODES[scale_mode]


def _flat(theta: torch.Tensor, format_id: int):
    lead, (nb, tpb) = theta.shape[:-2], theta.shape[-2:]
    if tpb != _TPB[FormatId(format_id)]:
        raise ValueError(f"expected blocks of {_TPB[FormatId(format_id)]} elements, got {tpb}")
    if theta.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("theta must be bf16 or fp32")
    m = math.prod(lead)
    return theta.reshape(m, nb * tpb).contiguous(), lead, m, nb, tpb


@torch.library.custom_op("cdl_b200::ecdl_quant_fwd", mutates_args=())
def ecdl_quant_fwd(theta: torch.Tensor, theta_kappa: torch.Tensor, seed: torch.Tensor, format_id: int,
                   theta_topk: int, scale_mode: str) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = _lib.require_cuda(theta, theta_kappa, seed)
    flat, lead, m, nb, tpb = _flat(theta, format_id)
    fp4 = FormatId(format_id) != FormatId.MXFP8
    cols = tpb // 2 if fp4 else tpb
    packed = torch.empty((m, nb * cols), dtype=torch.uint8, device=dev)
    scale = torch.empty((m, nb), dtype=torch.uint8, device=dev)
    alpha = torch.ones((), dtype=torch.float32, device=dev)
    ws = torch.empty(16, dtype=torch.uint8, device=dev)
    kappa = theta_kappa.detach().float().reshape(()).contiguous()
    _lib.call("cdlb200_ecdl_fwd", _lib.ptr(flat), int(flat.dtype == torch.float32), m, nb, int(format_id),
              _mode(scale_mode), _lib.ptr(kappa), _lib.ptr(seed), int(theta_topk), _lib.ptr(packed),
              _lib.ptr(scale), _lib.ptr(alpha), _lib.ptr(ws), _lib.stream(dev))
    packed = packed.reshape(*lead, nb, cols)
    if not fp4:
        packed = packed.view(torch.float8_e4m3fn)
    return packed, scale.reshape(*lead, nb, 1), alpha


@ecdl_quant_fwd.register_fake
def _(theta, theta_kappa, seed, format_id, theta_topk, scale_mode):
    lead, (nb, tpb) = theta.shape[:-2], theta.shape[-2:]
    fp4 = FormatId(format_id) != FormatId.MXFP8
    return (theta.new_empty((*lead, nb, tpb // 2 if fp4 else tpb), dtype=torch.uint8 if fp4 else torch.float8_e4m3fn),
            theta.new_empty((*lead, nb, 1), dtype=torch.uint8), theta.new_empty((), dtype=torch.float32))


@torch.library.custom_op("cdl_b200::ecdl_quant_bwd", mutates_args=())
def ecdl_quant_bwd(grad_proxy: torch.Tensor, theta: torch.Tensor, packed_scale: torch.Tensor,
                   kappa_backward: torch.Tensor, alpha: torch.Tensor, format_id: int, theta_topk: int,
                   scale_mode: str, need_dkappa: bool) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _lib.require_cuda(grad_proxy, theta, packed_scale, kappa_backward, alpha)
    flat, lead, m, nb, tpb = _flat(theta, format_id)
    g = grad_proxy.reshape(m, nb * tpb).to(flat.dtype).contiguous()
    dtheta = torch.empty_like(flat)
    scalars = torch.empty(2 if need_dkappa else 0, dtype=torch.float32, device=dev)
    nbytes = int(_lib.lib().cdlb200_ecdl_bwd_workspace_bytes(m, nb, int(format_id))) if need_dkappa else 0
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    kappa = kappa_backward.detach().float().reshape(()).contiguous()
    al = alpha.detach().float().reshape(()).contiguous()
    _lib.call("cdlb200_ecdl_bwd", _lib.ptr(g), _lib.ptr(flat), int(flat.dtype == torch.float32), m, nb,
              int(format_id), _lib.ptr(packed_scale.reshape(m, nb).contiguous()), _lib.ptr(kappa), _lib.ptr(al),
              int(theta_topk), _lib.ptr(dtheta), _lib.ptr(scalars) if need_dkappa else None, _lib.ptr(ws),
              ws.numel(), _lib.stream(dev))
    return dtheta, scalars


@ecdl_quant_bwd.register_fake
def _(grad_proxy, theta, packed_scale, kappa_backward, alpha, format_id, theta_topk, scale_mode, need_dkappa):
    m = math.prod(theta.shape[:-2])
    nb, tpb = theta.shape[-2:]
    return (theta.new_empty((m, nb * tpb)), theta.new_empty((2 if need_dkappa else 0,), dtype=torch.float32))


class EcdlQuantFn(torch.autograd.Function):
    """cdl/core/kernel/ecdl/autograd.py:102-158, on the B200 kernels."""

    @staticmethod
    def forward(ctx, theta, kappa_forward, kappa_backward, seed, format_id, theta_topk, scale_mode):
        seed.add_(1)
        packed_theta, packed_scale, alpha_eff = ecdl_quant_fwd(theta, kappa_forward, seed, format_id, theta_topk,
                                                               scale_mode)
        ctx.save_for_backward(theta, packed_scale, kappa_forward, kappa_backward, alpha_eff)
        ctx.format_id, ctx.theta_topk, ctx.scale_mode = format_id, theta_topk, scale_mode
        carrier = theta.new_zeros(()).expand(theta.shape)
        ctx.mark_non_differentiable(alpha_eff)
        return packed_theta, packed_scale, carrier, alpha_eff

    @staticmethod
    def backward(ctx, g_packed_theta, g_packed_scale, g_proxy, g_alpha_eff):
        theta, packed_scale, kappa_forward, kappa_backward, alpha_eff = ctx.saved_tensors
        coupled = kappa_backward is None  # the forward kappa also shapes the proxy and gets d(kappa)
        kappa_bwd = kappa_forward if coupled else kappa_backward
        need_dkappa = ctx.needs_input_grad[1] if coupled else ctx.needs_input_grad[2]
        dtheta, scalars = ecdl_quant_bwd(g_proxy.contiguous(), theta, packed_scale, kappa_bwd, alpha_eff,
                                         ctx.format_id, ctx.theta_topk, ctx.scale_mode, need_dkappa)
        dk_f = scalars[0].to(kappa_forward.dtype) if (coupled and need_dkappa) else None
        dk_b = scalars[0].to(kappa_backward.dtype) if ((not coupled) and need_dkappa) else None
        return dtheta.reshape(theta.shape), dk_f, dk_b, None, None, None, None


def ecdl_quant(theta, kappa_forward, kappa_backward, seed, format_id, theta_topk, scale_mode):
    return EcdlQuantFn.apply(theta, kappa_forward, kappa_backward, seed, int(format_id), theta_topk, scale_mode)


def nvfp4_ecdl_quant(theta, kappa_forward, kappa_backward, seed, theta_topk):
    return ecdl_quant(theta, kappa_forward, kappa_backward, seed, FormatId.NVFP4, theta_topk, "nvidia")


def mxfp4_ecdl_quant(theta, kappa_forward, kappa_backward, seed, theta_topk):
    return ecdl_quant(theta, kappa_forward, kappa_backward, seed, FormatId.MXFP4, theta_topk, "ocp")


def mxfp8_ecdl_quant(theta, kappa_forward, kappa_backward, seed, theta_topk):
    return ecdl_quant(theta, kappa_forward, kappa_backward, seed, FormatId.MXFP8, theta_topk, "ocp")
