"""The reference's own SmolLM2 NVFP4 QAT step on the GPU, from the unmodified
cdl package installed under ``baseline/_ref``.

Used by ``bench.py`` (the reference's step timed on the same box, beside this
library's) and by ``tests/test_loss_curve_gpu.py`` (loss-curve parity against
the reference's own step).  Nothing in ``cdl_b200`` imports it.

The step is the reference script's (``smollm2.py``):

* ``ModelController.apply_quant`` (smollm2.py:408-424): every
  ``q/k/v/o/gate/up/down_proj`` ``nn.Linear`` becomes a ``QLinear`` with
  ``SteQuant("nvfp4")`` on the activation and the weight and backend
  ``"native"`` (dequantize with the Triton kernels, bf16 matmul, STE;
  ``cdl/core/mm/native.py:6-17``); the script always sets ``"native"``, and
  cdl's ``"nvfp4"`` backend needs FlashInfer's ``b12x`` GEMM, built for
  sm_120 only;
* ``lm_loss`` (smollm2.py:667-677): Liger's fused linear cross entropy through
  the unquantized LM head;
* ``_step_optimizer`` (smollm2.py:638-659): ``clip_grad_norm_(1.0)`` then
  ``torch.optim.AdamW`` (betas (0.9, 0.95)); weight decay 0 and a constant
  learning rate, the BASELINE configs' settings, which this library's
  ``QatStep`` uses too.

The model is built exactly as ``cdl_b200.train.qat.build_model(...,
init_device="cpu")`` builds it (same ``LlamaConfig``, ``torch.manual_seed``,
CPU init, bf16), so both steps start from the same weights.
"""

from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def unavailable() -> str | None:
    """None when the reference package and its GPU dependencies import, else
    the reason, in one line."""
    if not os.path.isdir(os.path.join(REF, "cdl")):
        return "the reference package is not installed under baseline/_ref"
    if REF not in sys.path:
        sys.path.append(REF)
    try:
        import cdl.core.kernel.quant  # noqa: F401
        import cdl.model.components.linear  # noqa: F401
        import cdl.model.components.quant.ste  # noqa: F401
        from liger_kernel.transformers.functional import liger_fused_linear_cross_entropy  # noqa: F401
    except Exception as e:  # noqa: BLE001 - reported, not raised
        return f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"
    return None


def build_model(spec, device: torch.device, seed: int = 0) -> torch.nn.Module:
    """The random-init SmolLM2 of ``spec`` with the reference's quantized
    linears (``apply_quant``, smollm2.py:408-424)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from cdl.model.components.linear import QLinear
    from cdl.model.components.quant.ste import SteQuant

    cfg = LlamaConfig(
        vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
        num_hidden_layers=spec.layers, num_attention_heads=spec.heads, num_key_value_heads=spec.kv_heads,
        head_dim=spec.hidden // spec.heads, max_position_embeddings=spec.max_pos, rope_theta=spec.rope_theta,
        rms_norm_eps=1e-5, tie_word_embeddings=spec.tied, initializer_range=0.02, hidden_act="silu",
        attention_bias=False, mlp_bias=False, use_cache=False,
    )
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device("cpu"):
        model = LlamaForCausalLM(cfg)
    model = model.to(dtype=torch.bfloat16).to(device)
    with torch.no_grad():
        for name, module in list(model.named_modules()):
            parent_name, _, leaf = name.rpartition(".")
            if leaf not in TARGETS or not isinstance(module, torch.nn.Linear):
                continue
            parent = model.get_submodule(parent_name) if parent_name else model
            q = QLinear.from_linear(module)
            q.set_activation_quant(SteQuant("nvfp4"))
            q.set_weight_quant(SteQuant("nvfp4"))
            q.set_backend("native")
            setattr(parent, leaf, q)
    model.train()
    return model


class ReferenceQatStep:
    """One training step of the reference's script on ``device``."""

    def __init__(self, spec, device: torch.device, lr: float = 3e-4, seed: int = 0):
        reason = unavailable()
        if reason is not None:
            raise RuntimeError(reason)
        self.model = build_model(spec, device, seed)
        self.params = [p for p in self.model.parameters() if p.requires_grad]
        self.opt = torch.optim.AdamW(self.params, lr=lr, betas=(0.9, 0.95), weight_decay=0.0)

    def loss(self, input_ids: torch.Tensor) -> torch.Tensor:
        from liger_kernel.transformers.functional import liger_fused_linear_cross_entropy

        hidden = self.model.model(input_ids=input_ids, use_cache=False).last_hidden_state[:, :-1]
        targets = input_ids[:, 1:]
        return liger_fused_linear_cross_entropy(hidden.reshape(-1, hidden.shape[-1]), self.model.lm_head.weight,
                                                targets.reshape(-1), bias=self.model.lm_head.bias,
                                                reduction="mean")

    def step(self, input_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        loss = self.loss(input_ids)
        loss.backward()
        grad_norm = torch.nn.utils.clip_grad_norm_(self.params, 1.0)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach(), grad_norm.detach()
