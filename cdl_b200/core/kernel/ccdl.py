"""CCDL stochastic quantizer: the drop-in for ``cdl.core.kernel.ccdl``
(cdl/core/kernel/ccdl/autograd.py, launch.py) and the CCDL entry points of
``cdl.core.kernel`` (entries.py:10-76).

``ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, format_id,
theta_topk, q_topk)`` samples each block's scale from its learnable value q
on the scale grid (truncated window, ``q_kappa``) and each element's code as
ECDL does, and returns ``(packed_theta, packed_scale, carrier)``; the
backward gives theta its proxy gradient and q, both kappas and alpha theirs.
q is ``[..., nb]`` per theta row or one row ``[nb]`` (shape ``q.numel() ==
nb``) shared by all rows, as in the reference (layout.py:17-47).  Kernels:
``cdlb200_ccdl_fwd`` / ``cdlb200_ccdl_bwd`` (include/cdlb200_step.h).
"""

from __future__ import annotations

import math

import torch

from cdl_b200 import _lib
from cdl_b200.core.kernel.ecdl import FormatId, _flat


def _flatten_q(lead, nb: int, q: torch.Tensor):
    m = math.prod(lead)
    if q.numel() == nb:
        return q.reshape(1, nb).float().contiguous(), 0
    if q.numel() == m * nb:
        return q.reshape(m, nb).float().contiguous(), nb
    return (q * q.new_ones(*lead, nb, 1)).reshape(m, nb).float().contiguous(), nb


def reduce_q_grad(dq: torch.Tensor, theta: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Per-block q gradients back to the (possibly broadcast) shape of q."""
    full = dq.reshape(*theta.shape[:-2], -1)
    lead_pad = q.ndim - full.ndim - 1
    full = full.reshape((1,) * max(lead_pad, 0) + full.shape + (1,))
    dims = tuple(i for i, size in enumerate(q.shape) if size == 1 and full.shape[i] != 1)
    if dims:
        full = full.sum(dim=dims, keepdim=True)
    return full.reshape(q.shape)


def _scalar(t: torch.Tensor) -> torch.Tensor:
    return t.detach().float().reshape(()).contiguous()


@torch.library.custom_op("cdl_b200::ccdl_quant_fwd", mutates_args=())
def ccdl_quant_fwd(theta: torch.Tensor, q: torch.Tensor, theta_kappa: torch.Tensor, q_kappa: torch.Tensor,
                   alpha: torch.Tensor, seed: torch.Tensor, format_id: int, theta_topk: int,
                   q_topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _lib.require_cuda(theta, q, theta_kappa, q_kappa, alpha, seed)
    flat, lead, m, nb, tpb = _flat(theta, format_id)
    lq, qs = _flatten_q(lead, nb, q)
    fp4 = FormatId(format_id) != FormatId.MXFP8
    cols = tpb // 2 if fp4 else tpb
    packed = torch.empty((m, nb * cols), dtype=torch.uint8, device=dev)
    scale = torch.empty((m, nb), dtype=torch.uint8, device=dev)
    kt, kq, al = _scalar(theta_kappa), _scalar(q_kappa), _scalar(alpha)
    _lib.call("cdlb200_ccdl_fwd", _lib.ptr(flat), int(flat.dtype == torch.float32), m, nb, int(format_id),
              _lib.ptr(lq), qs, _lib.ptr(kt), _lib.ptr(kq), _lib.ptr(al), _lib.ptr(seed), int(theta_topk),
              int(q_topk), _lib.ptr(packed), _lib.ptr(scale), _lib.stream(dev))
    packed = packed.reshape(*lead, nb, cols)
    if not fp4:
        packed = packed.view(torch.float8_e4m3fn)
    scale = scale[:1].reshape(q.shape) if qs == 0 else scale.reshape(*lead, nb, 1)
    return packed, scale


@ccdl_quant_fwd.register_fake
def _(theta, q, theta_kappa, q_kappa, alpha, seed, format_id, theta_topk, q_topk):
    lead, (nb, tpb) = theta.shape[:-2], theta.shape[-2:]
    fp4 = FormatId(format_id) != FormatId.MXFP8
    shape = q.shape if q.numel() == nb else (*lead, nb, 1)
    return (theta.new_empty((*lead, nb, tpb // 2 if fp4 else tpb), dtype=torch.uint8 if fp4 else torch.float8_e4m3fn),
            theta.new_empty(shape, dtype=torch.uint8))


@torch.library.custom_op("cdl_b200::ccdl_quant_bwd", mutates_args=())
def ccdl_quant_bwd(grad_proxy: torch.Tensor, theta: torch.Tensor, q: torch.Tensor, packed_scale: torch.Tensor,
                   theta_kappa: torch.Tensor, q_kappa: torch.Tensor, alpha: torch.Tensor, format_id: int,
                   theta_topk: int, q_topk: int, need_dq: bool, need_dkt: bool, need_dkq: bool,
                   need_dal: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = _lib.require_cuda(grad_proxy, theta, q, packed_scale)
    flat, lead, m, nb, tpb = _flat(theta, format_id)
    lq, qs = _flatten_q(lead, nb, q)
    g = grad_proxy.reshape(m, nb * tpb).to(flat.dtype).contiguous()
    ps = packed_scale.reshape(-1, nb).contiguous()
    dtheta = torch.empty_like(flat)
    dq = torch.empty((m, nb) if need_dq else (0,), dtype=torch.float32, device=dev)
    need_scalars = need_dkt or need_dkq or need_dal
    scalars = torch.empty(3 if need_scalars else 0, dtype=torch.float32, device=dev)
    nbytes = int(_lib.lib().cdlb200_ccdl_bwd_workspace_bytes(m, nb, int(format_id))) if need_scalars else 0
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    kt, kq, al = _scalar(theta_kappa), _scalar(q_kappa), _scalar(alpha)
    _lib.call("cdlb200_ccdl_bwd", _lib.ptr(g), _lib.ptr(flat), int(flat.dtype == torch.float32), m, nb,
              int(format_id), _lib.ptr(lq), qs, _lib.ptr(ps), 0 if ps.shape[0] == 1 and m > 1 else nb,
              _lib.ptr(kt), _lib.ptr(kq), _lib.ptr(al), int(theta_topk), int(q_topk), _lib.ptr(dtheta),
              _lib.ptr(dq) if need_dq else None, _lib.ptr(scalars) if need_scalars else None, _lib.ptr(ws),
              ws.numel(), _lib.stream(dev))
    return dtheta, dq, scalars


@ccdl_quant_bwd.register_fake
def _(grad_proxy, theta, q, packed_scale, theta_kappa, q_kappa, alpha, format_id, theta_topk, q_topk, need_dq,
      need_dkt, need_dkq, need_dal):
    m = math.prod(theta.shape[:-2])
    nb, tpb = theta.shape[-2:]
    return (theta.new_empty((m, nb * tpb)), theta.new_empty((m, nb) if need_dq else (0,), dtype=torch.float32),
            theta.new_empty((3 if (need_dkt or need_dkq or need_dal) else 0,), dtype=torch.float32))


class CcdlQuantFn(torch.autograd.Function):
    """cdl/core/kernel/ccdl/autograd.py:118-180, on the B200 kernels."""

    @staticmethod
    def forward(ctx, theta, q, theta_kappa, q_kappa, alpha, seed, format_id, theta_topk, q_topk):
        seed.add_(1)
        packed_theta, packed_scale = ccdl_quant_fwd(theta, q, theta_kappa, q_kappa, alpha, seed, format_id,
                                                    theta_topk, q_topk)
        ctx.save_for_backward(theta, q, packed_scale, theta_kappa, q_kappa, alpha)
        ctx.format_id, ctx.topk = format_id, (theta_topk, q_topk)
        carrier = theta.new_zeros(()).expand(theta.shape)
        return packed_theta, packed_scale, carrier

    @staticmethod
    def backward(ctx, g_packed_theta, g_packed_scale, g_proxy):
        theta, q, packed_scale, theta_kappa, q_kappa, alpha = ctx.saved_tensors
        need_q, need_kt, need_kq, need_al = ctx.needs_input_grad[1:5]
        dtheta, dq, scalars = ccdl_quant_bwd(g_proxy.contiguous(), theta, q, packed_scale, theta_kappa, q_kappa,
                                             alpha, ctx.format_id, *ctx.topk, need_q, need_kt, need_kq, need_al)
        return (dtheta.reshape(theta.shape), reduce_q_grad(dq, theta, q).to(q.dtype) if need_q else None,
                scalars[0].to(theta_kappa.dtype).reshape(theta_kappa.shape) if need_kt else None,
                scalars[1].to(q_kappa.dtype).reshape(q_kappa.shape) if need_kq else None,
                scalars[2].to(alpha.dtype).reshape(alpha.shape) if need_al else None,
                None, None, None, None)


@torch.no_grad()
def ccdl_round(theta: torch.Tensor, q: torch.Tensor, alpha: torch.Tensor, format_id: int,
               level_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Deterministic CCDL quantize, cdl's ``cascaded_nearest_round``
    (cdl/core/ccdl.py:78-89) with format levels of ``level_dtype`` (bf16 or
    fp32), packed as the sampled forward packs: ``(packed [..., nb, cols],
    scale bytes shaped like the sampled forward's)``."""
    if level_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"ccdl_round: levels must be bf16 or fp32, got {level_dtype}")
    dev = _lib.require_cuda(theta, q, alpha)
    flat, lead, m, nb, tpb = _flat(theta, format_id)
    lq, qs = _flatten_q(lead, nb, q)
    fp4 = FormatId(format_id) != FormatId.MXFP8
    cols = tpb // 2 if fp4 else tpb
    packed = torch.empty((m, nb * cols), dtype=torch.uint8, device=dev)
    scale = torch.empty((m, nb), dtype=torch.uint8, device=dev)
    _lib.call("cdlb200_ccdl_round", _lib.ptr(flat), int(flat.dtype == torch.float32), m, nb, int(format_id),
              _lib.ptr(lq), qs, _lib.ptr(_scalar(alpha)), int(level_dtype == torch.bfloat16), _lib.ptr(packed),
              _lib.ptr(scale), _lib.stream(dev))
    packed = packed.reshape(*lead, nb, cols)
    if not fp4:
        packed = packed.view(torch.float8_e4m3fn)
    scale = scale[:1].reshape(q.shape) if qs == 0 else scale.reshape(*lead, nb, 1)
    return packed, scale


def ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, format_id, theta_topk, q_topk):
    return CcdlQuantFn.apply(theta, q, theta_kappa, q_kappa, alpha, seed, int(format_id), theta_topk, q_topk)


def nvfp4_ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, theta_topk, q_topk):
    return ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, FormatId.NVFP4, theta_topk, q_topk)


def mxfp4_ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, theta_topk, q_topk):
    return ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, FormatId.MXFP4, theta_topk, q_topk)


def mxfp8_ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, theta_topk, q_topk):
    return ccdl_quant(theta, q, theta_kappa, q_kappa, alpha, seed, FormatId.MXFP8, theta_topk, q_topk)
