"""SmolLM2 quantization-aware training step on the B200 path.

Mirrors what cdl's training driver does per micro-batch (smollm2.py:667-677
``lm_loss``, :638-659 ``_step_optimizer``, :408-424 ``apply_quant``): every
``q/k/v/o/gate/up/down_proj`` linear of a Llama decoder becomes a
``QLinear`` whose activation and weight pass through ``SteQuant`` (or one of
cdl's CCDL / ECDL quantizer variants) and whose matmul backend is ``nvfp4``
(or ``mxfp4`` / ``mxfp8`` / ``native``); the loss
is next-token cross entropy through the unquantized LM head, computed the way
cdl's Liger fused linear cross entropy does it (chunks of tokens; the logits
are never materialised for the whole batch, and the gradients of the hidden
states and of the head weight are formed in the same pass); the optimizer is
AdamW (betas 0.9/0.95) with gradient-norm clipping at 1.0, on CUDA both in
three launches of ``cdlb200_clip_adamw`` (``train/optim.py``).

Models are built from the BASELINE configurations with random init (std
0.02) -- no checkpoint is loaded -- and trained on uniform random tokens.

The options of cdl's script around the step are here too: LoRA and its
freeze policy, the warmup / cosine LR schedule, gradient accumulation, fp32
master weights, ``evaluate`` (perplexity) and ``run_training`` (its loop with
checkpoints and evaluation).

Data parallel: one process per GPU; ``train/dp.py``'s ``GradSync``
all-reduces (NCCL) each bf16 gradient from a backward hook while the backward
pass is still running, as torch's ``DistributedDataParallel`` would, and the
whole step -- all-reduces included -- is one CUDA graph, as on one GPU.  Each rank quantizes its own activations (per-rank amax, as a
single-GPU run would).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from cdl_b200 import _lib
from cdl_b200.model.components.linear import QLinear
from cdl_b200.model.components.quant.ste import SteQuant

QUANT_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True)
class ModelSpec:
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    intermediate: int
    vocab: int = 49152
    rope_theta: float = 10000.0
    tied: bool = True
    max_pos: int = 8192


SPECS = {
    # SmolLM2-135M
    "135m": ModelSpec("SmolLM2-135M", 30, 576, 9, 3, 1536, rope_theta=10000.0),
    # SmolLM2-1.7B
    "1.7b": ModelSpec("SmolLM2-1.7B", 24, 2048, 32, 32, 8192, rope_theta=130000.0),
    # small stand-in for tests
    "tiny": ModelSpec("tiny-llama", 2, 256, 4, 2, 512, vocab=1024, rope_theta=10000.0),
}


_CAUSAL_SDPA = "cdl_b200_causal_sdpa"


def _causal_attention() -> str:
    """transformers' SDPA attention registered under a name that has no mask
    builder: the model then passes no mask and SDPA runs with is_causal=True,
    which is the attention of independent, unpadded sequences -- the only
    inputs of this step.  It skips the packed-sequence probe of the mask
    builder, a device-to-host read on every forward."""
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    AttentionInterface.register(_CAUSAL_SDPA, sdpa_attention_forward)
    return _CAUSAL_SDPA


def build_model(spec: ModelSpec, device: torch.device, seed: int = 0, fused: bool | None = None,
                init_device: torch.device | str | None = None) -> nn.Module:
    """Random-init Llama of ``spec`` in bf16.  ``fused`` (default: on CUDA)
    routes its RMSNorm / rotary / SwiGLU through the fused kernels.  The
    weights are drawn on ``init_device`` (default ``device``) from
    ``torch.manual_seed(seed)``: with ``init_device="cpu"`` they are the ones a
    CPU run of the reference's script draws from the same seed."""
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(
        vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
        num_hidden_layers=spec.layers, num_attention_heads=spec.heads, num_key_value_heads=spec.kv_heads,
        head_dim=spec.hidden // spec.heads, max_position_embeddings=spec.max_pos, rope_theta=spec.rope_theta,
        rms_norm_eps=1e-5, tie_word_embeddings=spec.tied, initializer_range=0.02, hidden_act="silu",
        attention_bias=False, mlp_bias=False, use_cache=False,
    )
    cfg._attn_implementation = _causal_attention()
    torch.manual_seed(seed)
    with torch.device(init_device if init_device is not None else device):
        model = LlamaForCausalLM(cfg)
    model = model.to(dtype=torch.bfloat16).to(device)
    if fused if fused is not None else device.type == "cuda":
        from cdl_b200.model.components.fused import patch_llama

        patch_llama(model)
    return model


def untie_and_freeze(model: nn.Module, *, freeze_all: bool = True, train_head: bool = True) -> None:
    """cdl's parameter policy (smollm2.py:456-476, applied at :947-951 with
    ``freeze_all = use_lora or freeze_base`` and ``train_head = not use_lora
    and train_head``): the LM head gets its own copy of a tied embedding;
    then either everything but (optionally) the head is frozen, or only the
    input embedding (and, optionally, the head)."""
    embed, head = model.get_input_embeddings(), model.lm_head
    if head.weight is embed.weight:
        head.weight = nn.Parameter(embed.weight.detach().clone())
        model.config.tie_word_embeddings = False
    if not freeze_all:
        embed.weight.requires_grad_(False)
        if not train_head:
            head.weight.requires_grad_(False)
        return
    for p in model.parameters():
        p.requires_grad_(False)
    if train_head:
        head.weight.requires_grad_(True)


def lr_lambda(warmup_steps: int = 0, lr_decay: str = "constant", max_steps: int = 0, min_lr_ratio: float = 0.1):
    """cdl's learning-rate factor (smollm2.py:599-610): linear warmup to 1,
    then constant or a cosine down to ``min_lr_ratio`` at ``max_steps``."""
    if lr_decay not in ("constant", "cosine"):
        raise ValueError(f"unknown lr_decay {lr_decay!r}")

    def f(step: int) -> float:
        if step < warmup_steps:
            return (step + 1) / warmup_steps
        if lr_decay == "cosine" and max_steps > warmup_steps:
            progress = min(1.0, (step - warmup_steps) / (max_steps - warmup_steps))
            return min_lr_ratio + 0.5 * (1.0 - min_lr_ratio) * (1.0 + math.cos(math.pi * progress))
        return 1.0

    return f


def _cdl_variants() -> dict:
    """cdl's quantizer variants (smollm2.py:86-135): name -> (family, activation class, weight class)."""
    from cdl_b200.model.components.quant import ccdl, ecdl

    return {
        "nvfp4_ccdl": ("ccdl", ccdl.Nvfp4CascadedCdlQuantForActivation, ccdl.Nvfp4CascadedCdlQuantForWeight),
        "mxfp4_ccdl": ("ccdl", ccdl.Mxfp4CascadedCdlQuantForActivation, ccdl.Mxfp4CascadedCdlQuantForWeight),
        "mxfp8_ccdl": ("ccdl", ccdl.Mxfp8CascadedCdlQuantForActivation, ccdl.Mxfp8CascadedCdlQuantForWeight),
        "nvfp4_ecdl": ("ecdl", ecdl.Nvfp4ExtendedCdlQuantForActivation, ecdl.Nvfp4ExtendedCdlQuantForWeight),
        "mxfp4_ecdl": ("ecdl", ecdl.Mxfp4ExtendedCdlQuantForActivation, ecdl.Mxfp4ExtendedCdlQuantForWeight),
        "mxfp8_ecdl": ("ecdl", ecdl.Mxfp8ExtendedCdlQuantForActivation, ecdl.Mxfp8ExtendedCdlQuantForWeight),
    }


def build_activation_quant(variant: str, in_features: int, sim: str, dtype: torch.dtype = torch.bfloat16, *,
                           kappa: float = 2.0, kappa_bwd: float | None = None, theta_topk: int = 5,
                           q_topk: int = 5, kernel: str = "triton"):
    """cdl's ``_build_activation_quant`` (smollm2.py:352-374): "none", "ste"
    (``sim`` is the STE format) or a CDL variant over inputs shaped
    ``(1, in_features)``."""
    from cdl_b200.model.components.quant.identity import IdentityQuant

    if variant == "none":
        return IdentityQuant()
    if variant == "ste":
        return SteQuant(sim)
    family, act_cls, _ = _cdl_variants()[variant]
    if family == "ccdl":
        return act_cls((1, in_features), theta_topk, q_topk, dtype, kappa, kernel=kernel)
    return act_cls((1, in_features), theta_topk, dtype, kappa, kappa_bwd, kernel=kernel)


def build_weight_quant(variant: str, weight: torch.Tensor, sim: str, dtype: torch.dtype = torch.bfloat16, *,
                       kappa: float = 2.0, kernel: str = "triton"):
    """cdl's ``_build_weight_quant`` (smollm2.py:377-397), on the weight's device."""
    from cdl_b200.model.components.quant.identity import IdentityQuant

    if variant == "none":
        return IdentityQuant()
    if variant == "ste":
        return SteQuant(sim)
    _, _, w_cls = _cdl_variants()[variant]
    return w_cls(weight.detach(), dtype, kappa, kernel=kernel).to(weight.device)


def apply_quant(model: nn.Module, backend: str = "nvfp4", simulation: str | None = None, *,
                activation: str = "ste", weight: str = "ste", dtype: torch.dtype = torch.bfloat16,
                activation_kappa: float = 2.0, activation_kappa_bwd: float | None = None,
                weight_kappa: float = 2.0, theta_topk: int = 5, q_topk: int = 5, kernel: str = "triton",
                lora: tuple[int, int] | None = None) -> int:
    """Swap every target nn.Linear for a QLinear (smollm2.py:408-424) with
    cdl's quantizer variants: ``activation`` / ``weight`` each "none", "ste"
    or one of ``{nvfp4,mxfp4,mxfp8}_{ccdl,ecdl}``; ``lora = (r, alpha)``
    adds cdl's merged LoRA adapter to each (the weight quantizer then sees
    ``W + alpha / r * B A``).

    ``backend="none"`` leaves the model unquantized (bf16 reference runs)."""
    if backend == "none":
        return 0
    names = ("none", "ste", *_cdl_variants())
    if activation not in names or weight not in names:
        raise ValueError(f"unknown quantizer variant {activation!r} / {weight!r}")
    base = backend.split("_")[0]  # "nvfp4_qbwd" quantizes like "nvfp4"
    sim = simulation or (base if base.startswith("mx") else "nvfp4")
    count = 0
    for name, module in list(model.named_modules()):
        parent_name, _, leaf = name.rpartition(".")
        if leaf not in QUANT_TARGETS or not isinstance(module, nn.Linear):
            continue
        parent = model.get_submodule(parent_name) if parent_name else model
        q = QLinear.from_linear(module)
        if lora is not None:
            q.set_lora(*lora)
        q.set_activation_quant(build_activation_quant(activation, q.in_features, sim, dtype,
                                                      kappa=activation_kappa, kappa_bwd=activation_kappa_bwd,
                                                      theta_topk=theta_topk, q_topk=q_topk,
                                                      kernel=kernel).to(q.weight.device))
        q.set_weight_quant(build_weight_quant(weight, q.weight, sim, dtype, kappa=weight_kappa, kernel=kernel))
        q.set_backend(backend)
        setattr(parent, leaf, q)
        count += 1
    return count


class LinearCrossEntropy(torch.autograd.Function):
    """Mean cross entropy of ``h @ w^T`` against ``targets``, ``chunk`` tokens
    at a time (the algorithm of Liger's fused linear cross entropy, which cdl
    uses for its LM head, smollm2.py:667-677).  Per chunk: logits in the
    hidden dtype, their fp32 log-sum-exp and the loss, then
    ``d loss / d logits = (softmax - onehot) / n`` in the hidden dtype,
    ``grad_h = dl @ w`` and ``grad_w += dl^T @ h``.  The backward only scales
    the stored gradients."""

    @staticmethod
    def forward(ctx, h: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, chunk: int) -> torch.Tensor:
        n = h.shape[0]
        grad_h = torch.empty_like(h) if ctx.needs_input_grad[0] else None
        grad_w = torch.zeros_like(w) if ctx.needs_input_grad[1] else None
        # on the GPU one kernel per chunk (cdlb200_cross_entropy) turns the
        # bf16 logits into per-row losses and, in place, the bf16 gradient
        kernel = h.is_cuda and h.dtype == torch.bfloat16 and w.shape[0] % 8 == 0
        if kernel:
            targets = targets.to(torch.int64).contiguous()
            rows_loss = torch.empty(n, dtype=torch.float32, device=h.device)
            inv_n = float(np.float32(1.0) / np.float32(n))
        else:
            total = torch.zeros((), dtype=torch.float32, device=h.device)
        for s in range(0, n, chunk):
            hc, tc = h[s:s + chunk], targets[s:s + chunk]
            if kernel:
                dl = hc @ w.t()
                _lib.call("cdlb200_cross_entropy", _lib.ptr(dl), _lib.ptr(tc), dl.shape[0], dl.shape[1], inv_n,
                          _lib.ptr(rows_loss) + 4 * s, _lib.stream(h.device))
            else:
                logits = (hc @ w.t()).float()
                lse = torch.logsumexp(logits, dim=1)
                total += (lse - logits.gather(1, tc[:, None])[:, 0]).sum()
                p = logits.sub_(lse[:, None]).exp_()
                p[torch.arange(p.shape[0], device=p.device), tc] -= 1.0
                dl = p.div_(n).to(h.dtype)
            if grad_h is not None:
                torch.mm(dl, w, out=grad_h[s:s + chunk])
            if grad_w is not None:
                grad_w.addmm_(dl.t(), hc)
        ctx.save_for_backward(grad_h, grad_w)
        if kernel:
            total = rows_loss.sum()
        return total / n

    @staticmethod
    def backward(ctx, grad_loss: torch.Tensor):
        grad_h, grad_w = ctx.saved_tensors
        gl = grad_loss.to(grad_h.dtype if grad_h is not None else grad_w.dtype)
        grads = [g for g in (grad_h, grad_w) if g is not None]
        if all(g.is_cuda and g.dtype == torch.bfloat16 and g.is_contiguous() and g.numel() % 8 == 0 for g in grads):
            # scaled in place by the value read on the device (no work when it
            # is 1: the loss's own backward); the stored gradients are used
            # once, this backward being the only reader
            gl = gl.reshape(1).contiguous()
            for g in grads:
                _lib.call("cdlb200_scale_bf16", _lib.ptr(g), g.numel(), _lib.ptr(gl), _lib.stream(g.device))
            return grad_h, grad_w, None, None
        return (grad_h * gl if grad_h is not None else None, grad_w * gl if grad_w is not None else None, None, None)


def lm_loss(model: nn.Module, input_ids: torch.Tensor, chunk: int = 2048) -> torch.Tensor:
    """Mean next-token cross entropy through the LM head (smollm2.py:667-677)."""
    hidden = model.model(input_ids=input_ids, use_cache=False).last_hidden_state[:, :-1]
    h = hidden.reshape(-1, hidden.shape[-1])
    targets = input_ids[:, 1:].reshape(-1)
    if chunk <= 0:  # plain path: full fp32 logits
        return F.cross_entropy(model.lm_head(h).float(), targets, reduction="mean")
    w = model.lm_head.weight
    if not torch.is_grad_enabled():  # evaluation: no gradient buffers in the chunk loop
        h, w = h.detach(), w.detach()
    return LinearCrossEntropy.apply(h, w, targets, chunk)


@torch.no_grad()
def evaluate(model: nn.Module, loader, device: torch.device) -> float:
    """Perplexity over ``loader``'s batches of token ids (smollm2.py:681-694):
    exp of the token-weighted mean loss, in eval mode (deterministic
    quantizers).  The sum stays on the device until the end."""
    was_training = model.training
    model.eval()
    total = torch.zeros((), dtype=torch.float64, device=device)
    tokens = 0
    try:
        for input_ids in loader:
            input_ids = input_ids.to(device, non_blocking=True)
            n = input_ids.numel() - input_ids.shape[0]
            total += lm_loss(model, input_ids).double() * n
            tokens += n
    finally:
        model.train(was_training)
    return math.exp(float(total) / tokens)


class LossModule(nn.Module):
    """Model + loss as one module, so data parallelism wraps the whole forward."""

    def __init__(self, model: nn.Module):
        super().__init__()
        self.model = model

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return lm_loss(self.model, input_ids)


def flops_per_token(spec: ModelSpec, seq: int) -> float:
    """6 * params + 12 * layers * hidden * seq (training FLOPs per token)."""
    h, L = spec.hidden, spec.layers
    kvd = spec.kv_heads * (h // spec.heads)
    per_layer = h * h * 2 + 2 * h * kvd + 3 * h * spec.intermediate
    params = L * per_layer + spec.vocab * h * (1 if spec.tied else 2)
    return 6.0 * params + 12.0 * L * h * seq


class QatStep:
    """One QAT training step: forward, loss, backward (+ DP all-reduce), clip, AdamW."""

    def __init__(self, spec: ModelSpec, device: torch.device, backend: str = "nvfp4", lr: float = 3e-4,
                 grad_clip: float = 1.0, seed: int = 0, ddp: bool = False,
                 fused: bool | None = None, graph: bool = False, optimizer: str | None = None,
                 activation: str = "ste", weight: str = "ste", quant_lr: float = 3e-4, train_alpha: bool = True,
                 train_kappa: bool = False, use_lora: bool = False, lora_r: int = 8, lora_alpha: int = 16,
                 freeze_base: bool = False, train_head: bool = True, untie: bool = False, warmup_steps: int = 0,
                 lr_decay: str = "constant", max_steps: int = 0, min_lr_ratio: float = 0.1,
                 fp32_master_weights: bool = False, init_device: torch.device | str | None = None,
                 comm_sms: int | None = None, **quant_options):
        self.spec = spec
        self.device = device
        self.backend = backend
        self.model = build_model(spec, device, seed, fused, init_device)
        # the BASELINE configs train every parameter with tied embeddings;
        # cdl's script unties the head and applies its freeze policy
        if untie or use_lora or freeze_base:
            untie_and_freeze(self.model, freeze_all=use_lora or freeze_base,
                             train_head=not use_lora and train_head)
        self.n_quant = apply_quant(self.model, backend, activation=activation, weight=weight,
                                   lora=(lora_r, lora_alpha) if use_lora else None, **quant_options)
        self.model.train()
        on_cuda = device.type == "cuda"
        # the CDL quantizers' own parameters (fp32 log scales / temperatures)
        # form one more AdamW group at quant_lr, as cdl's build_optimizer
        # does (smollm2.py:555-604); the optimizer is then torch's AdamW
        from cdl_b200.model.components.quant.ccdl import CascadedCdlQuantMixin
        from cdl_b200.model.components.quant.ecdl import ExtendedCdlQuantMixin

        cg, cp = CascadedCdlQuantMixin.cascaded_cdl_get_param_groups(self.model, quant_lr, train_alpha, train_kappa)
        eg, ep = ExtendedCdlQuantMixin.extended_cdl_get_param_groups(self.model, quant_lr, train_kappa)
        quant_ids = {id(p) for p in cp | ep}
        quant_params = [p for g in cg + eg for p in g["params"]]
        params = [p for p in self.model.parameters() if p.requires_grad]
        self.params = params
        decay = [p for p in params if p.ndim > 1 and id(p) not in quant_ids]
        no_decay = [p for p in params if p.ndim <= 1 and id(p) not in quant_ids]
        # "fused": clip + AdamW through cdlb200_clip_adamw (CUDA, bf16
        # parameters only); "torch": clip_grad_norm_ + torch.optim.AdamW with
        # its default (foreach) implementation, as cdl constructs it
        self.optimizer = optimizer or ("fused" if on_cuda and not quant_ids and not fp32_master_weights else "torch")
        if self.optimizer == "fused" and fp32_master_weights:
            raise ValueError("fp32 master weights need optimizer='torch'")
        if self.optimizer == "fused" and quant_ids:
            raise ValueError("the fused optimizer takes bf16 parameters only; CDL quantizers need optimizer='torch'")
        # fp32 master copies of the non-fp32 parameters, which the optimizer
        # updates and copies back (smollm2.py:570-575, 649-657)
        self.master_pairs: list[tuple[nn.Parameter, nn.Parameter]] = []

        def opt_param(p):
            if fp32_master_weights and p.dtype != torch.float32:
                m = nn.Parameter(p.detach().float().clone())
                self.master_pairs.append((p, m))
                return m
            return p

        if fp32_master_weights:
            decay, no_decay = [opt_param(p) for p in decay], [opt_param(p) for p in no_decay]
            quant_params = [opt_param(p) for p in quant_params]
        if self.optimizer == "fused":
            from cdl_b200.train.optim import ClipAdamW

            # the QLinear weights of the nvfp4 backends are re-encoded by the
            # step that updates them: with the dequantized copy the bf16
            # backward reads (nvfp4), or with the encoding of w^T the quantized
            # dgrad reads (nvfp4_qbwd)
            qls = [m for m in self.model.modules() if isinstance(m, QLinear) and isinstance(m.weight_quant, SteQuant)]
            encode = [m.weight for m in qls if m.backend == "nvfp4"]
            encode_dual = [m.weight for m in qls if m.backend == "nvfp4_qbwd"]
            self.opt = ClipAdamW(params, lr=lr, betas=(0.9, 0.95), weight_decay=0.0, max_norm=grad_clip,
                                 encode=encode, encode_dual=encode_dual)
        elif self.optimizer == "torch":
            groups = [{"params": decay, "weight_decay": 0.0}, {"params": no_decay, "weight_decay": 0.0},
                      {"params": quant_params, "lr": quant_lr, "weight_decay": 0.0}]
            self.opt = torch.optim.AdamW([g for g in groups if g["params"]], lr=lr, betas=(0.9, 0.95),
                                         capturable=graph and on_cuda)
        else:
            raise ValueError(f"unknown optimizer {optimizer!r}")
        schedule = warmup_steps > 0 or lr_decay != "constant"
        if schedule and graph:
            raise ValueError("a learning-rate schedule needs eager steps (a captured step keeps its lr)")
        self.lr_scheduler = (torch.optim.lr_scheduler.LambdaLR(
            self.opt, lr_lambda(warmup_steps, lr_decay, max_steps, min_lr_ratio)) if schedule else None)
        self.graph_mode = graph and on_cuda
        self._graph = None
        self.grad_clip = grad_clip
        self.net = LossModule(self.model)
        # data parallel: gradients averaged over ranks from backward hooks
        # (train/dp.py), capturable in the step's CUDA graph
        self.sync = None
        # data parallel on CUDA: SMs the backward pass's persistent kernels
        # (the GEMMs, the dual encoder) leave to NCCL's all-reduce kernels,
        # which would otherwise queue behind kernels that hold every SM
        self.comm_sms = 0
        if ddp:
            from cdl_b200.train.dp import GradSync

            self.sync = GradSync(params)
            if on_cuda:
                self.comm_sms = 16 if comm_sms is None else int(comm_sms)
                self._sms = torch.cuda.get_device_properties(device).multi_processor_count

    def check_status(self) -> None:
        """Raise ``CdlB200Error`` if a kernel of this step recorded a timed-out
        bounded wait (a GEMM, or the one-launch NVFP4 quantizer's grid
        barrier) since the last check.  Reads device memory: call it between
        steps, outside a timed region."""
        if self.device.type == "cuda":
            _lib.check_status(self.device)

    @torch.no_grad()
    def calibrate(self, samples) -> None:
        """Initialize the CCDL activation quantizers' scales from calibration
        batches of token ids, on the native backend, as cdl's
        ``init_activation_q`` does (smollm2.py:478-491)."""
        from cdl_b200.model.components.quant.ccdl import CascadedCdlQuantMixin

        qls = [m for m in self.model.modules() if isinstance(m, QLinear)]
        for m in qls:
            m.set_backend("native")
        try:
            CascadedCdlQuantMixin.cascaded_cdl_init_act_q_pass(self.model, list(samples))
        finally:
            for m in qls:
                m.set_backend(self.backend)

    def _backward(self, loss: torch.Tensor, scale: float, last: bool) -> None:
        """``(loss * scale).backward()``; data parallel: the gradients are
        summed over ranks, the loss pre-scaled by 1 / world, after the last
        micro-batch only (the earlier ones accumulate locally)."""
        if self.sync is None:
            (loss * scale if scale != 1.0 else loss).backward()
            return
        self.sync.begin(reduce=last)
        cap = self.comm_sms > 0 and last
        if cap:
            _lib.set_persistent_sm_limit(max(self._sms - self.comm_sms, 2))
        try:
            (loss * (scale * self.sync.loss_scale)).backward()
        finally:
            if cap:
                _lib.set_persistent_sm_limit(0)
            self.sync.finish()

    def _eager_step(self, input_ids) -> tuple[torch.Tensor, torch.Tensor]:
        if self.device.type != "cuda":
            return self._step_body(input_ids)
        # the fused kernels' amax words come from one buffer zeroed once per step
        from cdl_b200.model.components import fused

        fused.begin_step(self.device)
        try:
            return self._step_body(input_ids)
        finally:
            fused.end_step()

    def _step_body(self, input_ids) -> tuple[torch.Tensor, torch.Tensor]:
        if isinstance(input_ids, torch.Tensor):
            loss = self.net(input_ids)
            self._backward(loss, 1.0, True)
        else:  # gradient accumulation over micro-batches, as cdl's loop (smollm2.py:816-851)
            micro = list(input_ids)
            n = len(micro)
            if n == 0:
                raise ValueError("no micro-batches")
            loss = None
            for j, ids in enumerate(micro):
                part = self.net(ids)
                self._backward(part, 1.0 / n if n > 1 else 1.0, j == n - 1)
                part = part.detach() / n if n > 1 else part.detach()
                loss = part if loss is None else loss + part
        if self.optimizer == "fused":
            gnorm = self.opt.step()
        else:
            gnorm = torch.nn.utils.clip_grad_norm_(self.params, self.grad_clip, foreach=True)
            if self.master_pairs:
                with torch.no_grad():
                    for p, m in self.master_pairs:
                        if p.grad is not None:
                            m.grad = p.grad.float()
                    self.opt.step()
                    for p, m in self.master_pairs:
                        p.copy_(m)
                        m.grad = None
            else:
                self.opt.step()
        if self.lr_scheduler is not None:
            self.lr_scheduler.step()
        if self.master_pairs:  # the optimizer holds the masters: clear the model's gradients
            for p in self.params:
                p.grad = None
        else:
            self.opt.zero_grad(set_to_none=True)
        return loss.detach(), gnorm.detach()

    def step(self, input_ids) -> tuple[torch.Tensor, torch.Tensor]:
        """One training step on a batch of token ids, or on a list of
        micro-batches whose gradients are accumulated (each loss divided by
        their count; with data parallelism the gradients are averaged over
        ranks after the last one) before one optimizer step; the returned
        loss is their mean.  In graph
        mode (one batch per step) the first call runs warm-up steps
        on a side stream and captures the whole step (forward, backward,
        clipping, AdamW) in a CUDA graph; every call then copies the tokens
        into the graph's input buffer and replays it.  The returned loss and
        gradient norm are the graph's output buffers."""
        if not self.graph_mode:
            return self._eager_step(input_ids)
        if not isinstance(input_ids, torch.Tensor):
            raise ValueError("graph mode takes one batch per step")
        if self._graph is None:
            self._capture(input_ids)
        self._static_ids.copy_(input_ids, non_blocking=True)
        self._graph.replay()
        return self._static_out

    def _capture(self, input_ids: torch.Tensor, warmup: int = 3) -> None:
        self._static_ids = input_ids.detach().clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._eager_step(self._static_ids)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._graph = torch.cuda.CUDAGraph()
        launches0 = _lib.launches
        # data parallel: the NCCL process group's watchdog thread may query
        # the events of the warm-up all-reduces while this thread captures;
        # a thread-local capture keeps its calls legal (the all-reduces
        # issued from the backward hooks are captured on their streams)
        mode = "thread_local" if self.sync is not None else "global"
        with torch.cuda.graph(self._graph, capture_error_mode=mode):
            self._static_out = self._eager_step(self._static_ids)
        # kernels of this library in the captured step (each replay runs them all)
        self.graph_launches = _lib.launches - launches0

    def release_graph(self) -> None:
        """Drop the captured step.  A graph that holds NCCL collectives must
        be released before the process group is destroyed."""
        if self._graph is not None:
            torch.cuda.synchronize(self.device)
            self._graph = None
            self._static_out = None


def run_training(step: QatStep, train_batches, *, epochs: int = 1, grad_accum_steps: int = 1, max_steps: int = 0,
                 start_step: int = 0, test_batches=None, eval_every: int = 0, save_every: int = 0,
                 checkpoint_path=None, log_every: int = 0, log=None) -> int:
    """cdl's training loop (smollm2.py:777-930) around a ``QatStep``:
    ``grad_accum_steps`` batches per optimizer step (a shorter window at the
    end of an epoch), stop at ``max_steps``, resume by skipping the batches
    of ``start_step`` steps, a checkpoint every ``save_every`` steps and at
    the end (``cdl_b200.train.checkpoint``), perplexity on ``test_batches``
    every ``eval_every`` steps and at the end.  ``train_batches`` is
    re-iterated each epoch (a ``DeviceBlockLoader`` or any iterable of token
    batches); ``log(step, loss, grad_norm, lr)`` runs every ``log_every``
    steps (its arguments are device tensors but ``lr``).  Returns the global
    step reached."""
    from cdl_b200.train.checkpoint import save_checkpoint

    def save(epoch, gs):
        if checkpoint_path is not None:
            save_checkpoint(checkpoint_path, step.model, step.opt, step.lr_scheduler, epoch, gs)

    n_batches = len(train_batches)
    per_epoch = -(-n_batches // grad_accum_steps)
    start_epoch = min(start_step // per_epoch, epochs - 1) if per_epoch else 0
    skip = max(start_step - start_epoch * per_epoch, 0) * grad_accum_steps
    gs, last_saved, last_eval, epoch = start_step, -1, -1, start_epoch
    for epoch in range(start_epoch, epochs):
        step.model.train()
        window: list = []
        it = iter(train_batches)
        for i, ids in enumerate(it):
            if i < skip:
                continue
            if not window:
                width = min(grad_accum_steps, n_batches - i)
            window.append(ids)
            if len(window) < width:
                continue
            loss, gnorm = step.step(window if len(window) > 1 else window[0])
            window = []
            gs += 1
            if log is not None and log_every > 0 and gs % log_every == 0:
                log(gs, loss, gnorm, step.opt.param_groups[0]["lr"])
            if save_every > 0 and gs % save_every == 0:
                save(epoch, gs)
                last_saved = gs
            if test_batches is not None and eval_every > 0 and gs % eval_every == 0:
                ppl = evaluate(step.model, test_batches, step.device)
                last_eval = gs
                if log is not None:
                    log(gs, None, None, ppl)
            if max_steps and gs >= max_steps:
                break
        skip = 0
        if max_steps and gs >= max_steps:
            break
    if gs != last_saved:
        save(min(epoch, epochs - 1), gs)
    if test_batches is not None and gs != last_eval:
        ppl = evaluate(step.model, test_batches, step.device)
        if log is not None:
            log(gs, None, None, ppl)
    return gs


def random_tokens(batch: int, seq: int, vocab: int, seed: int, device: torch.device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), generator=g, device=device)


def expected_initial_loss(spec: ModelSpec) -> float:
    return math.log(spec.vocab)
