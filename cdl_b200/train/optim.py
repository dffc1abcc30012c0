"""Gradient clipping + AdamW of the QAT step in three CUDA launches.

cdl's training step (smollm2.py) runs ``torch.nn.utils.clip_grad_norm_``
and then ``torch.optim.AdamW``: a norm pass over every gradient, an in-place
multiply of every gradient by the clip coefficient and the optimizer pass,
each a chain of multi-tensor launches.  ``ClipAdamW`` does the same
arithmetic through ``cdlb200_clip_adamw`` (include/cdlb200_step.h): one
sum-of-squares pass, one single-CTA finalize (per-tensor bf16 norms, total
norm, clip coefficient, bias corrections, all on the device), one update pass
that applies the coefficient on the fly.  No host synchronization, so the
step can be captured in a CUDA graph.
"""

from __future__ import annotations

import ctypes
from typing import Iterable

import torch

from cdl_b200 import _lib


class ClipAdamW:
    """``clip_grad_norm_(params, max_norm, foreach=True)`` followed by
    ``AdamW(params, lr, betas, eps, weight_decay).step()`` for bf16 CUDA
    parameters; moments are bf16 as torch keeps them for bf16 parameters.
    ``step()`` returns the total gradient norm (a 0-d fp32 tensor holding the
    bf16 value torch's clip returns).  Parameters whose ``grad`` is None are
    skipped, as torch does."""

    def __init__(self, params: Iterable[torch.Tensor], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, max_norm: float = 1.0):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("ClipAdamW: no parameters")
        dev = self.params[0].device
        for p in self.params:
            if p.device != dev or not p.is_cuda:
                raise ValueError("ClipAdamW: all parameters must be on one CUDA device")
            if p.dtype != torch.bfloat16 or not p.is_contiguous() or p.numel() % 8 or p.data_ptr() % 16:
                raise ValueError("ClipAdamW: parameters must be contiguous bf16, numel % 8 == 0, 16-byte aligned")
        self.lr, self.betas, self.eps, self.weight_decay, self.max_norm = lr, betas, eps, weight_decay, max_norm
        self.exp_avg = [torch.zeros_like(p) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p) for p in self.params]
        self._table = (_lib.AdamwTensor * len(self.params))()
        for i, p in enumerate(self.params):
            t = self._table[i]
            t.param, t.exp_avg, t.exp_avg_sq = p.data_ptr(), self.exp_avg[i].data_ptr(), self.exp_avg_sq[i].data_ptr()
            t.numel = p.numel()
        self._numel = [p.numel() for p in self.params]
        nbytes = int(_lib.lib().cdlb200_clip_adamw_workspace_bytes(ctypes.addressof(self._table), len(self.params)))
        self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self._norm = torch.zeros((), dtype=torch.float32, device=dev)
        self.device = dev

    @torch.no_grad()
    def step(self) -> torch.Tensor:
        tab = self._table
        for i, p in enumerate(self.params):
            g = p.grad
            if g is None:
                tab[i].grad, tab[i].numel = None, 0
                continue
            if g.dtype != torch.bfloat16 or not g.is_contiguous():
                raise ValueError("ClipAdamW: gradients must be contiguous bf16")
            tab[i].grad, tab[i].numel = g.data_ptr(), self._numel[i]
        b1, b2 = self.betas
        _lib.call("cdlb200_clip_adamw", ctypes.addressof(tab), len(self.params), float(self.max_norm),
                  float(self.lr), float(b1), float(b2), float(self.eps), float(self.weight_decay),
                  _lib.ptr(self._ws), self._ws.numel(), _lib.ptr(self._norm), _lib.stream(self.device))
        return self._norm.clone()

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    @property
    def steps_done(self) -> int:
        """Completed steps (reads the device counter: synchronizes)."""
        return int(self._ws[:4].view(torch.float32).item())
