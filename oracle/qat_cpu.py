"""CPU NVFP4 QAT step -- TEST INFRASTRUCTURE ONLY (bench.py's CPU baseline
and reference arm).

The reference's training step with its ``native`` backend, restated for the
host cores: every ``q/k/v/o/gate/up/down_proj`` linear of a random-init
SmolLM2 quantizes its activation and its weight to NVFP4 on every forward
(``SteQuant("nvfp4")``, ``cdl/model/components/quant/ste.py:25-31``; the
codes, scales and alpha come from this package's C oracle, the restatement of
cdl's torch nearest-round path), dequantizes both
(``cdl/core/kernel/dequant.py:43-47``) and multiplies them in bf16 with the
straight-through estimator (``cdl/core/mm/native.py:6-17``: the gradients
are ``g @ deq(w)`` and ``g^T @ deq(x)``); the loss is the mean next-token
cross entropy of the fp32 upcast of the bf16 LM-head logits (the arithmetic
of the Liger loss of ``smollm2.py:667-677``); then ``clip_grad_norm_(1.0)``
and ``torch.optim.AdamW`` (betas 0.9/0.95, lr 3e-4; ``smollm2.py:638-659``).

The oracle runs on row chunks of each tensor in a thread pool (ctypes
releases the GIL); the NVFP4 global amax is reduced over all chunks first.
"""

from __future__ import annotations

import concurrent.futures
import time

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

import oracle

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class _Pool:
    ex: concurrent.futures.ThreadPoolExecutor | None = None
    threads = 1


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def nvfp4_fake_quant(t: torch.Tensor) -> torch.Tensor:
    """bf16 ``deq(Q(t))`` of a 2-D bf16 tensor through the C oracle."""
    x = _bits(t)
    n = max(1, min(_Pool.threads, x.shape[0]))
    chunks = np.array_split(np.arange(x.shape[0]), n)
    gmax = max(_Pool.ex.map(lambda idx: oracle.nvfp4_global(x[idx[0]: idx[-1] + 1])[0], chunks))
    alpha = np.float32(gmax) * (np.float32(1.0) / np.float32(2688.0))  # quant.py:96-101, as on the device
    outs = list(_Pool.ex.map(lambda idx: oracle.quant(x[idx[0]: idx[-1] + 1], oracle.NVFP4, gmax)[:2], chunks))
    deq = list(_Pool.ex.map(lambda ps: oracle.dequant(ps[0], ps[1], oracle.NVFP4, np.array([alpha], np.float32)),
                            outs))
    return torch.from_numpy(np.concatenate(deq).view(np.int16)).view(torch.bfloat16).reshape(t.shape)


class _NativeNvfp4(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        xd, wd = nvfp4_fake_quant(x), nvfp4_fake_quant(w)
        ctx.save_for_backward(xd, wd)
        return xd @ wd.t()

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        xd, wd = ctx.saved_tensors
        return g @ wd, g.t() @ xd


class OracleQLinear(nn.Module):
    """``QLinear`` with ``SteQuant("nvfp4")`` on both inputs and the native backend."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        self.weight = linear.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        return _NativeNvfp4.apply(x2, self.weight).reshape(*x.shape[:-1], -1)


def apply_oracle_quant(model: nn.Module) -> int:
    n = 0
    for name, module in list(model.named_modules()):
        parent_name, _, leaf = name.rpartition(".")
        if leaf in TARGETS and isinstance(module, nn.Linear):
            parent = model.get_submodule(parent_name) if parent_name else model
            setattr(parent, leaf, OracleQLinear(module))
            n += 1
    return n


def qat_step_rate(spec, batch: int, seq: int, threads: int, steps: int = 1, full_tokens: int | None = None):
    """Time ``steps`` CPU NVFP4 QAT steps of ``spec`` on ``batch x seq`` tokens.

    Returns ``(tokens_per_s, description)``.  With ``full_tokens`` the step
    time is also split into the per-step weight quantize / dequantize (a
    fixed cost per step) and the rest (per token), and the rate is projected
    to a step of ``full_tokens`` tokens."""
    from cdl_b200 import workloads
    from cdl_b200.train.qat import build_model

    torch.set_num_threads(threads)
    _Pool.threads = threads
    _Pool.ex = concurrent.futures.ThreadPoolExecutor(threads)
    try:
        model = build_model(spec, torch.device("cpu"), seed=0, fused=False)
        apply_oracle_quant(model)
        model.train()
        params = [p for p in model.parameters() if p.requires_grad]
        opt = torch.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.0)
        batches = list(workloads.token_batches(batch, seq, spec.vocab, 0, steps))
        t0 = time.perf_counter()
        for ids in batches:
            hidden = model.model(input_ids=ids, use_cache=False).last_hidden_state[:, :-1]
            h = hidden.reshape(-1, hidden.shape[-1])
            loss = F.cross_entropy((h @ model.lm_head.weight.t()).float(), ids[:, 1:].reshape(-1))
            loss.backward()
            torch.nn.utils.clip_grad_norm_(params, 1.0)
            opt.step()
            opt.zero_grad(set_to_none=True)
        dt = (time.perf_counter() - t0) / steps
        tokens = batch * seq
        desc = (f"{steps} CPU NVFP4 QAT step(s) of {spec.name} on {batch}x{seq} tokens ({threads} threads): "
                f"reference native-backend numerics -- NVFP4 quantize/dequantize of every linear's activation and "
                f"weight per forward (C oracle of cdl's torch path), bf16 matmuls with the STE, fp32 cross "
                f"entropy, clip + torch AdamW; {dt:.2f} s per step")
        if full_tokens is None:
            return tokens / dt, desc
        # the per-step fixed cost: quantize + dequantize of every weight (timed once more)
        ws = [m.weight for m in model.modules() if isinstance(m, OracleQLinear)]
        t1 = time.perf_counter()
        for w in ws:
            nvfp4_fake_quant(w)
        fixed = time.perf_counter() - t1
        per_token = max(dt - fixed, 0.0) / tokens
        proj = fixed + per_token * full_tokens
        return full_tokens / proj, (desc + f"; of which {fixed:.2f} s weight quantize/dequantize per step; projected "
                                           f"to {full_tokens} tokens per step: {proj:.1f} s")
    finally:
        _Pool.ex.shutdown()
        _Pool.ex = None
