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
from torch.autograd.graph import increment_version

from cdl_b200 import _lib

# attribute of an encoded weight: (version, packed, scales, alpha, dequantized
# or None[, packed of w^T, scales of w^T])
ENCODED_ATTR = "_cdlb200_nvfp4"


class ClipAdamW(torch.optim.Optimizer):
    """``clip_grad_norm_(params, max_norm, foreach=True)`` followed by
    ``AdamW(params, lr, betas, eps, weight_decay).step()`` for bf16 CUDA
    parameters; moments are bf16 as torch keeps them for bf16 parameters.
    ``step()`` returns the total gradient norm (a 0-d fp32 tensor holding the
    bf16 value torch's clip returns).  Parameters whose ``grad`` is None are
    skipped, as torch does.

    A ``torch.optim.Optimizer`` with one parameter group, so torch's LR
    schedulers drive it (``lr``, ``betas``, ``eps`` and ``weight_decay`` are
    read from the group at every step; a step captured in a CUDA graph keeps
    the values of the capture).  ``state_dict()`` / ``load_state_dict()`` use
    ``torch.optim.AdamW``'s layout (per-parameter ``step``, ``exp_avg``,
    ``exp_avg_sq``), so checkpoints move between the two."""

    def __init__(self, params: Iterable[torch.Tensor], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0, max_norm: float = 1.0,
                 encode: Iterable[torch.Tensor] = (), encode_dual: Iterable[torch.Tensor] = ()):
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("ClipAdamW: no parameters")
        dev = params[0].device
        for p in params:
            if p.device != dev or not p.is_cuda:
                raise ValueError("ClipAdamW: all parameters must be on one CUDA device")
            if p.dtype != torch.bfloat16 or not p.is_contiguous() or p.numel() % 8 or p.data_ptr() % 16:
                raise ValueError("ClipAdamW: parameters must be contiguous bf16, numel % 8 == 0, 16-byte aligned")
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay, amsgrad=False,
                        maximize=False, foreach=None, capturable=False, differentiable=False, fused=None)
        super().__init__(params, defaults)
        self.params = params
        self.max_norm = max_norm
        self.exp_avg = [torch.zeros_like(p) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p) for p in self.params]
        self._table = (_lib.AdamwTensor * len(self.params))()
        for i, p in enumerate(self.params):
            t = self._table[i]
            t.param, t.exp_avg, t.exp_avg_sq = p.data_ptr(), self.exp_avg[i].data_ptr(), self.exp_avg_sq[i].data_ptr()
            t.numel = p.numel()
            self.state[p] = {"exp_avg": self.exp_avg[i], "exp_avg_sq": self.exp_avg_sq[i]}
        self._numel = [p.numel() for p in self.params]
        nbytes = int(_lib.lib().cdlb200_clip_adamw_workspace_bytes(ctypes.addressof(self._table), len(self.params)))
        self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self._norm = torch.zeros((), dtype=torch.float32, device=dev)
        self.device = dev
        encode, encode_dual = list(encode), list(encode_dual)
        self._encoders = ([WeightEncoder(self, encode)] if encode else []) + (
            [WeightEncoder(self, encode_dual, dual=True)] if encode_dual else [])

    @property
    def lr(self) -> float:
        return self.param_groups[0]["lr"]

    @lr.setter
    def lr(self, value: float) -> None:
        self.param_groups[0]["lr"] = value

    @torch.no_grad()
    def step(self, closure=None) -> torch.Tensor:
        if closure is not None:
            raise ValueError("ClipAdamW: closures are not supported")
        tab = self._table
        for i, p in enumerate(self.params):
            g = p.grad
            if g is None:
                tab[i].grad, tab[i].numel = None, 0
                continue
            if g.dtype != torch.bfloat16 or not g.is_contiguous():
                raise ValueError("ClipAdamW: gradients must be contiguous bf16")
            tab[i].grad, tab[i].numel = g.data_ptr(), self._numel[i]
        group = self.param_groups[0]
        b1, b2 = group["betas"]
        _lib.call("cdlb200_clip_adamw", ctypes.addressof(tab), len(self.params), float(self.max_norm),
                  float(group["lr"]), float(b1), float(b2), float(group["eps"]), float(group["weight_decay"]),
                  _lib.ptr(self._ws), self._ws.numel(), _lib.ptr(self._norm), _lib.stream(self.device))
        # the kernels wrote the parameters in place: advance their version
        # counters as a torch in-place update would
        increment_version([p for i, p in enumerate(self.params) if tab[i].numel])
        for enc in self._encoders:
            enc.refresh()
        return self._norm.clone()

    @property
    def steps_done(self) -> int:
        """Completed steps (reads the device counter: synchronizes)."""
        return int(self._ws[:4].view(torch.float32).item())

    def state_dict(self) -> dict:
        """AdamW's layout; ``step`` is a CPU fp32 tensor as AdamW keeps it
        (reads the device counter: synchronizes)."""
        sd = super().state_dict()
        step = torch.tensor(float(self.steps_done), dtype=torch.float32)
        for st in sd["state"].values():
            st["step"] = step.clone()
        return sd

    def load_state_dict(self, state_dict: dict) -> None:
        """Accepts this optimizer's or ``torch.optim.AdamW``'s state_dict with
        one parameter group over the same parameters: copies the moments into
        the buffers the kernels use and sets the step counter."""
        super().load_state_dict(state_dict)
        step = 0.0
        for i, p in enumerate(self.params):
            st = self.state.get(p, {})
            if "exp_avg" in st:
                self.exp_avg[i].copy_(st["exp_avg"])
                self.exp_avg_sq[i].copy_(st["exp_avg_sq"])
            else:  # never stepped in the saved run
                self.exp_avg[i].zero_()
                self.exp_avg_sq[i].zero_()
            if "step" in st:
                step = max(step, float(st["step"]))
            self.state[p] = {"exp_avg": self.exp_avg[i], "exp_avg_sq": self.exp_avg_sq[i]}
        self._ws[:4].view(torch.float32).fill_(step)


class WeightEncoder:
    """NVFP4 encodings of the quantized linears' weights, refreshed by the
    optimizer step that changed them.

    cdl quantizes every weight in each forward and dequantizes it again for
    the bf16 dgrad GEMM of the backward (core/mm/nvfp4.py).  The weights only
    change in the optimizer step, so here the update kernel also folds each
    weight's new max|w| into an amax word, and right after it one launch
    writes, for every weight, the codes, the GEMM-layout scales, alpha and
    either the dequantized copy the bf16 backward reads
    (``cdlb200_nvfp4_encode_multi``) or, with ``dual``, the encoding of
    ``w^T`` the quantized dgrad GEMM reads (``cdlb200_nvfp4_dual_multi``) --
    the same values the per-layer quantize and dequantize would produce.
    Each weight carries them as ``ENCODED_ATTR`` together with its version;
    the linear layer uses them while the version matches (see ``SteTensor``),
    else it quantizes as usual.  Weights that do not fit the encoder's layout
    (rows % 128 and (k/16) % 4; with ``dual`` rows and k multiples of 64) are
    left to the per-layer path."""

    def __init__(self, opt: ClipAdamW, weights: list[torch.Tensor], dual: bool = False):
        index = {id(p): i for i, p in enumerate(opt.params)}
        self.opt = opt
        self.dual = dual
        fits = ((lambda w: w.shape[0] % 64 == 0 and w.shape[1] % 64 == 0) if dual
                else (lambda w: w.shape[0] % 128 == 0 and w.shape[1] % 64 == 0))
        self.weights = [w for w in weights if id(w) in index and w.dim() == 2 and fits(w)]
        dev = opt.device
        n = len(self.weights)
        self.amax = torch.zeros(max(n, 1), dtype=torch.int32, device=dev)
        self.table = ((_lib.Nvfp4DualTensor if dual else _lib.Nvfp4EncodeTensor) * max(n, 1))()
        self.buffers = []
        for j, w in enumerate(self.weights):
            rows, k = w.shape
            packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=dev)
            scale = torch.empty((rows + 127) // 128 * 128, k // 16, dtype=torch.uint8, device=dev)
            alpha = torch.empty(1, dtype=torch.float32, device=dev)
            amax_ptr = self.amax.data_ptr() + 4 * j
            t = self.table[j]
            if dual:
                tpacked = torch.empty(k, rows // 2, dtype=torch.uint8, device=dev)
                tscale = torch.empty((k + 127) // 128 * 128, rows // 16, dtype=torch.uint8, device=dev)
                t.x, t.rows, t.cols, t.amax, t.amax_words, t.alpha = w.data_ptr(), rows, k, amax_ptr, 1, alpha.data_ptr()
                t.row_packed, t.row_scale = packed.data_ptr(), scale.data_ptr()
                t.col_packed, t.col_scale = tpacked.data_ptr(), tscale.data_ptr()
                self.buffers.append((packed, scale, alpha, None, tpacked, tscale))
            else:
                deq = torch.empty(rows, k, dtype=torch.bfloat16, device=dev)
                t.x, t.rows, t.k, t.amax, t.amax_words = w.data_ptr(), rows, k, amax_ptr, 1
                t.packed, t.scale, t.alpha, t.deq = packed.data_ptr(), scale.data_ptr(), alpha.data_ptr(), deq.data_ptr()
                self.buffers.append((packed, scale, alpha, deq))
            opt._table[index[id(w)]].amax = amax_ptr

    def refresh(self) -> None:
        """Encode the weights the last update wrote (those that had a grad)."""
        opt = self.opt
        live = []
        for j, w in enumerate(self.weights):
            if w.grad is None:  # not updated this step: keep (or lack) its encoding
                self.table[j].rows = 0
            else:
                self.table[j].rows = w.shape[0]
                live.append(j)
        if not live:
            return
        fn = "cdlb200_nvfp4_dual_multi" if self.dual else "cdlb200_nvfp4_encode_multi"
        _lib.call(fn, ctypes.addressof(self.table), len(self.weights), _lib.stream(opt.device))
        for j in live:
            w = self.weights[j]
            setattr(w, ENCODED_ATTR, (w._version, *self.buffers[j]))
