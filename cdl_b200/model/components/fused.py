"""Fused RMSNorm, rotary embedding and SwiGLU for the Llama decoder of the
QAT step (``include/cdlb200_step.h``).

cdl trains SmolLM2 as a Hugging Face ``LlamaForCausalLM`` (smollm2.py), whose
``LlamaRMSNorm``, ``apply_rotary_pos_emb`` and ``LlamaMLP`` run as chains of
eager elementwise kernels.  ``patch_llama(model)`` swaps them for one CUDA
pass each (forward and backward), keeping the rounding steps of the eager
modules.  Tensors that are not bf16 on a CUDA device go through the original
Hugging Face code.  The RMSNorm and SwiGLU outputs feed quantized linears;
their kernels also produce the output's global amax (``AMAX_ATTR``), so the
NVFP4 quantize of those activations is a single encode pass; the SwiGLU and
rotary backward kernels do the same for the gradients of the gate / up and
q / k projections (``grad_amax``).
"""

from __future__ import annotations

import types
import weakref

import torch

from cdl_b200 import _lib


# attribute of a kernel output carrying the NVFP4 global amax formed in its
# epilogue: (amax word, version of the output when it was written)
AMAX_ATTR = "_cdlb200_amax"


def attach_amax(t: torch.Tensor, amax: torch.Tensor) -> None:
    setattr(t, AMAX_ATTR, (amax, t._version))


# Gradients reach the next autograd node as views made by the engine (the
# reshape of a linear's output), not as the tensor the kernel wrote, so their
# amax words are found by address: (weak reference to the written gradient,
# amax words, its version when written).  While the gradient is alive no
# other tensor can share its address, and the version check rejects it once
# something wrote into it.
_GRAD_AMAX: list = []
_GRAD_AMAX_MAX = 8


def attach_grad_amax(t: torch.Tensor, amax: torch.Tensor) -> None:
    _GRAD_AMAX.insert(0, (weakref.ref(t), amax, t._version))
    del _GRAD_AMAX[_GRAD_AMAX_MAX:]


def grad_amax(g: torch.Tensor) -> torch.Tensor | None:
    """The amax words of gradient ``g`` (the tensor a kernel wrote or a view
    of all of it) if its producer formed them, else None."""
    for ref, amax, version in _GRAD_AMAX:
        t = ref()
        if (t is not None and t.data_ptr() == g.data_ptr() and t.numel() == g.numel() and t.device == g.device
                and g._version == version and g.is_contiguous()):
            return amax
    return None


class _AmaxArena:
    """The amax words of one training step, handed out from one buffer that
    the step zeroes with a single fill when it begins (in place of a
    zero-filled allocation per kernel call: ~190 fills per 1.7B step).
    Outside a step, or once the buffer is used up, every call gets fresh
    zero-filled words.  Words handed out in a step are valid until the next
    step begins."""

    SLOTS = 4096

    def __init__(self):
        self.buf = None
        self.used = 0
        self.active = False


_ARENA = _AmaxArena()


def begin_step(device: torch.device) -> None:
    """Zero the step's amax words (one fill) and hand them out until end_step."""
    a = _ARENA
    if a.buf is None or a.buf.device != device:
        a.buf = torch.empty(a.SLOTS, _lib.AMAX_WORDS, dtype=torch.int32, device=device)
    a.buf.zero_()
    a.used = 0
    a.active = True


def end_step() -> None:
    _ARENA.active = False


def new_amax(device: torch.device, rows: int | None = None) -> torch.Tensor:
    """Zeroed amax words: [AMAX_WORDS], or [rows, AMAX_WORDS]."""
    n = 1 if rows is None else rows
    a = _ARENA
    if a.active and a.buf.device == device and a.used + n <= a.SLOTS:
        words = a.buf[a.used:a.used + n]
        a.used += n
        return words[0] if rows is None else words
    shape = (_lib.AMAX_WORDS,) if rows is None else (rows, _lib.AMAX_WORDS)
    return torch.zeros(shape, dtype=torch.int32, device=device)


def _cuda_bf16(*ts: torch.Tensor) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        d = x.shape[-1]
        x2 = x.reshape(-1, d).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        amax = new_amax(x.device)
        _lib.call("cdlb200_rmsnorm_fwd", _lib.ptr(x2), _lib.ptr(w), x2.shape[0], d, float(eps), _lib.ptr(y),
                  _lib.ptr(rstd), _lib.ptr(amax), _lib.stream(x.device))
        attach_amax(y, amax)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2, w, rstd = ctx.saved_tensors
        rows, d = x2.shape
        dy2 = dy.reshape(rows, d).contiguous()
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        nbytes = int(_lib.lib().cdlb200_rmsnorm_bwd_workspace_bytes(rows, d))
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x2.device)
        _lib.call("cdlb200_rmsnorm_bwd", _lib.ptr(dy2), _lib.ptr(x2), _lib.ptr(w), _lib.ptr(rstd), rows, d,
                  _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(ws), ws.numel(), _lib.stream(x2.device))
        return dx.view(ctx.shape), dw, None


class ResidualRMSNormFn(torch.autograd.Function):
    """``h = res + x`` (bf16) and ``y = RMSNorm(h)`` in one pass: the decoder's
    residual add and the norm after it.  The backward returns one gradient for
    both inputs -- the norm's input gradient plus the gradient ``h`` receives
    from its other consumer, summed in the kernel as autograd would sum them
    -- and forms its amax: it is the gradient of the o / down projection that
    produced ``x``, which the quantized backward encodes."""

    @staticmethod
    def forward(ctx, res: torch.Tensor, x: torch.Tensor, w: torch.Tensor, eps: float):
        d = x.shape[-1]
        r2 = res.reshape(-1, d).contiguous()
        x2 = x.reshape(-1, d).contiguous()
        h = torch.empty_like(x2)
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        amax = new_amax(x.device)
        _lib.call("cdlb200_add_rmsnorm_fwd", _lib.ptr(r2), _lib.ptr(x2), _lib.ptr(w), x2.shape[0], d, float(eps),
                  _lib.ptr(h), _lib.ptr(y), _lib.ptr(rstd), _lib.ptr(amax), _lib.stream(x.device))
        attach_amax(y, amax)
        ctx.save_for_backward(h, w, rstd)
        ctx.shape = x.shape
        return h.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, dh: torch.Tensor | None, dy: torch.Tensor | None):
        h, w, rstd = ctx.saved_tensors
        rows, d = h.shape
        dy2 = (dy if dy is not None else torch.zeros(ctx.shape, dtype=h.dtype, device=h.device))
        dy2 = dy2.reshape(rows, d).contiguous()
        dh2 = dh.reshape(rows, d).contiguous() if dh is not None else None
        dx = torch.empty_like(h)
        dw = torch.empty_like(w)
        amax = new_amax(h.device)
        nbytes = int(_lib.lib().cdlb200_rmsnorm_bwd_workspace_bytes(rows, d))
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=h.device)
        _lib.call("cdlb200_rmsnorm_bwd_add", _lib.ptr(dy2), _lib.ptr(h), _lib.ptr(w), _lib.ptr(rstd), _lib.ptr(dh2),
                  rows, d, _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(amax), _lib.ptr(ws), ws.numel(),
                  _lib.stream(h.device))
        attach_grad_amax(dx, amax)
        g = dx.view(ctx.shape)
        return g, g, dw, None


class RopeFn(torch.autograd.Function):
    """``x * cos + rotate_half(x) * sin`` on ``x[B, H, S, D]`` (a transposed
    view of the ``[B, S, H, D]`` projection output), ``cos/sin[Bc, S, D]``
    with ``Bc`` 1 or B."""

    @staticmethod
    def _run(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, backward: int) -> torch.Tensor:
        xt = x.transpose(1, 2)
        if not xt.is_contiguous():
            xt = xt.contiguous()
        b, s, h, d = xt.shape
        out = torch.empty_like(xt)
        # the backward's output is the q / k projection's gradient: form its amax
        amax = new_amax(x.device) if backward else None
        _lib.call("cdlb200_rope", _lib.ptr(xt), _lib.ptr(cos), _lib.ptr(sin), b * s, h, d, cos.shape[0] * s,
                  backward, _lib.ptr(out), _lib.ptr(amax), _lib.stream(x.device))
        if amax is not None:
            attach_grad_amax(out, amax)
        return out.transpose(1, 2)

    @staticmethod
    def forward(ctx, x, cos, sin):
        ctx.save_for_backward(cos, sin)
        return RopeFn._run(x, cos, sin, 0)

    @staticmethod
    def backward(ctx, g):
        cos, sin = ctx.saved_tensors
        return RopeFn._run(g, cos, sin, 1), None, None


class SwiGLUFn(torch.autograd.Function):
    """``silu(g) * u`` with both rounded to bf16, as ``LlamaMLP`` computes it."""

    @staticmethod
    def forward(ctx, g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
        g, u = g.contiguous(), u.contiguous()
        h = torch.empty_like(g)
        amax = new_amax(g.device)
        _lib.call("cdlb200_swiglu_fwd", _lib.ptr(g), _lib.ptr(u), g.numel(), _lib.ptr(h), _lib.ptr(amax),
                  _lib.stream(g.device))
        attach_amax(h, amax)
        ctx.save_for_backward(g, u)
        return h

    @staticmethod
    def backward(ctx, dh: torch.Tensor):
        g, u = ctx.saved_tensors
        dh = dh.contiguous()
        dg, du = torch.empty_like(g), torch.empty_like(u)
        amax = new_amax(g.device, 2)
        _lib.call("cdlb200_swiglu_bwd", _lib.ptr(dh), _lib.ptr(g), _lib.ptr(u), g.numel(), _lib.ptr(dg), _lib.ptr(du),
                  _lib.ptr(amax[0]), _lib.ptr(amax[1]), _lib.stream(g.device))
        attach_grad_amax(dg, amax[0])
        attach_grad_amax(du, amax[1])
        return dg, du


def _rmsnorm_forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
    d = hidden_states.shape[-1]
    if _cuda_bf16(hidden_states, self.weight) and d % 8 == 0 and d <= 2048:
        return RMSNormFn.apply(hidden_states, self.weight, self.variance_epsilon)
    return self._cdlb200_eager_forward(hidden_states)


def _mlp_forward(self, x: torch.Tensor) -> torch.Tensor:
    g, u = self.gate_proj(x), self.up_proj(x)
    if _cuda_bf16(g, u) and g.numel() % 8 == 0 and self.config.hidden_act == "silu":
        return self.down_proj(SwiGLUFn.apply(g, u))
    return self.down_proj(self.act_fn(g) * u)


_EAGER_ROPE = None


def _apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1):
    if (unsqueeze_dim == 1 and _cuda_bf16(q, k, cos, sin) and q.shape[-1] % 16 == 0 and cos.dim() == 3
            and cos.is_contiguous() and sin.is_contiguous() and cos.shape[0] in (1, q.shape[0])):
        return RopeFn.apply(q, cos, sin), RopeFn.apply(k, cos, sin)
    return _EAGER_ROPE(q, k, cos, sin, unsqueeze_dim)


def _llama_model_forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                         inputs_embeds=None, use_cache=None, **kwargs):
    """``LlamaModel.forward`` with each residual add fused into the RMSNorm
    that follows it: the two adds of a decoder layer become
    ``h = x + attn(norm1(x)); y = norm2(h)`` and ``x' = h + mlp(y);
    y' = norm1'(x')`` (the next layer's input norm, or the final norm) --
    the same operations in the same order as transformers' loop
    (``LlamaDecoderLayer.forward``), one pass each.  Inputs the fused path does
    not cover (a mask, a cache, embeddings not bf16 on a GPU) take the
    original forward."""
    from transformers.modeling_outputs import BaseModelOutputWithPast

    layers = self.layers[: self.config.num_hidden_layers]
    fused = (attention_mask is None and past_key_values is None and not use_cache and len(layers) > 0
             and self.config.hidden_size % 8 == 0 and self.config.hidden_size <= 2048)
    if fused:
        embeds = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        fused = _cuda_bf16(embeds, self.norm.weight)
    if not fused:
        return self._cdlb200_eager_forward(input_ids=input_ids, attention_mask=attention_mask,
                                           position_ids=position_ids, past_key_values=past_key_values,
                                           inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
    if position_ids is None:
        position_ids = torch.arange(embeds.shape[1], device=embeds.device).unsqueeze(0)
    pos = self.rotary_emb(embeds, position_ids=position_ids)
    x, y = embeds, layers[0].input_layernorm(embeds)
    for i, layer in enumerate(layers):
        a, _ = layer.self_attn(hidden_states=y, attention_mask=None, position_ids=position_ids, past_key_values=None,
                               use_cache=False, position_embeddings=pos, **kwargs)
        norm2 = layer.post_attention_layernorm
        h, y = ResidualRMSNormFn.apply(x, a, norm2.weight, norm2.variance_epsilon)
        m = layer.mlp(y)
        nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else self.norm
        x, y = ResidualRMSNormFn.apply(h, m, nxt.weight, nxt.variance_epsilon)
    return BaseModelOutputWithPast(last_hidden_state=y, past_key_values=None)


def patch_llama(model: torch.nn.Module, fuse_residual: bool = True) -> int:
    """Route the RMSNorm, rotary and SwiGLU parts of a transformers Llama model
    through the fused kernels, and (``fuse_residual``) its decoder loop through
    the residual-add + RMSNorm kernels; returns the number of modules
    patched."""
    global _EAGER_ROPE
    from transformers.models.llama import modeling_llama as ml

    if _EAGER_ROPE is None:
        _EAGER_ROPE = ml.apply_rotary_pos_emb
        ml.apply_rotary_pos_emb = _apply_rotary_pos_emb
    count = 0
    for m in model.modules():
        if isinstance(m, ml.LlamaRMSNorm) and not hasattr(m, "_cdlb200_eager_forward"):
            m._cdlb200_eager_forward = m.forward
            m.forward = types.MethodType(_rmsnorm_forward, m)
            count += 1
        elif isinstance(m, ml.LlamaMLP) and not getattr(m, "_cdlb200_fused", False):
            m.forward = types.MethodType(_mlp_forward, m)
            m._cdlb200_fused = True
            count += 1
        elif (fuse_residual and isinstance(m, ml.LlamaModel) and not hasattr(m, "_cdlb200_eager_forward")
              and all(type(layer) is ml.LlamaDecoderLayer for layer in m.layers)):
            m._cdlb200_eager_forward = m.forward
            m.forward = types.MethodType(_llama_model_forward, m)
            count += 1
    return count
