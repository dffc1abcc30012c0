"""Generate the reference loss curve for the QAT loss-curve parity test.

Runs the REFERENCE's own training-step code on the CPU -- cdl's ``QLinear``
(``cdl/model/components/linear.py:14-103``) with ``SteQuant("nvfp4")`` on the
activation and the weight (``cdl/model/components/quant/ste.py:13-89``) and
the ``native`` backend (dequantize, then bf16 matmul with the STE,
``cdl/core/mm/native.py:6-17``) on every ``q/k/v/o/gate/up/down_proj`` of a
random-init SmolLM2 (``smollm2.py:408-424``), the mean next-token cross
entropy through the unquantized LM head (``smollm2.py:667-677``), gradient
clipping at 1.0 and ``torch.optim.AdamW`` with betas (0.9, 0.95), weight
decay 0 and lr 3e-4 (``smollm2.py:555-604, 638-659``) -- and records the loss
and the gradient norm of every step in ``loss_curve_<spec>.json``.

Two substitutions, because the reference's GPU kernels cannot run on a CPU:

* ``nvfp4_quant`` / ``nvfp4_dequant`` (Triton) are replaced by the
  reference's torch nearest-round path with fp32 format tables
  (``cdl/core/ecdl.py:115-131``, the same function ``make_golden.py`` uses:
  bit-identical codes and scales) and its dequantize order
  (``cdl/core/kernel/dequant.py:43-47``);
* Liger's fused linear cross entropy (CUDA only) is replaced by
  ``F.cross_entropy`` on the fp32 upcast of the bf16 logits, which is the
  arithmetic Liger performs.

The model is built on the CPU from ``torch.manual_seed(seed)`` and cast to
bf16; the token batches come from ``cdl_b200.workloads.token_batches``.  The
GPU test builds the same model (CPU init, then moved) and feeds the same
batches.

Usage: ``python tests/golden/make_loss_curve.py --reference <cdl/src>
[--spec 135m --batch 1 --seq 256 --steps 200]``.  Needs the reference
checkout; the committed output does not.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from cdl_b200 import workloads  # noqa: E402

E2M1_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)


def torch_path_nvfp4_quant(x: torch.Tensor, block_chunk: int = 32):
    from make_golden import NVFP4, ref_quant

    packed, scale, alpha, _ = ref_quant(x.to(torch.bfloat16), NVFP4)
    return packed, scale, alpha


def torch_path_nvfp4_dequant(packed: torch.Tensor, scale: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """bf16((e2m1 * e4m3 scale) * alpha), element 2j in the low nibble."""
    rows = packed.shape[0]
    lo, hi = packed & 0xF, packed >> 4
    nib = torch.stack([lo, hi], dim=-1).reshape(rows, -1).long()
    val = E2M1_MAG[nib & 7] * torch.where(nib >= 8, -1.0, 1.0)
    sc = scale.contiguous().view(torch.float8_e4m3fn).float()
    val = val.reshape(rows, scale.shape[1], 16) * sc[..., None]
    return (val * alpha.float()).reshape(rows, -1).to(torch.bfloat16)


def build_reference_model(spec, seed: int):
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
    model = LlamaForCausalLM(cfg).to(dtype=torch.bfloat16)
    targets = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"}
    with torch.no_grad():  # as the reference's apply_quant (smollm2.py:408)
        _swap(model, targets, QLinear, SteQuant)
    return model


def _swap(model, targets, QLinear, SteQuant) -> None:
    for name, module in list(model.named_modules()):
        parent_name, _, leaf = name.rpartition(".")
        if leaf not in targets or not isinstance(module, torch.nn.Linear):
            continue
        parent = model.get_submodule(parent_name) if parent_name else model
        q = QLinear.from_linear(module)
        q.set_activation_quant(SteQuant("nvfp4"))
        q.set_weight_quant(SteQuant("nvfp4"))
        q.set_backend("native")
        setattr(parent, leaf, q)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CDL_REFERENCE_SRC", ""))
    ap.add_argument("--spec", default="135m")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <path to the cdl checkout's src directory>")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(args.threads)

    import cdl.model.components.quant.ste as ste
    from cdl_b200.train.qat import SPECS

    ste.nvfp4_quant = torch_path_nvfp4_quant
    ste.nvfp4_dequant = torch_path_nvfp4_dequant

    spec = SPECS[args.spec]
    model = build_reference_model(spec, args.seed)
    model.train()
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.0)
    losses, gnorms = [], []
    t0 = time.time()
    for step, ids in enumerate(workloads.token_batches(args.batch, args.seq, spec.vocab, args.seed, args.steps)):
        hidden = model.model(input_ids=ids, use_cache=False).last_hidden_state[:, :-1]
        h = hidden.reshape(-1, hidden.shape[-1])
        logits = h @ model.lm_head.weight.t()
        loss = F.cross_entropy(logits.float(), ids[:, 1:].reshape(-1), reduction="mean")
        loss.backward()
        gnorm = torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss))
        gnorms.append(float(gnorm))
        print(f"step {step} loss {losses[-1]:.6f} gnorm {gnorms[-1]:.4f} ({time.time() - t0:.0f} s)", flush=True)
    out = {
        "spec": args.spec, "batch": args.batch, "seq": args.seq, "steps": args.steps, "seed": args.seed,
        "backend": "reference native (cdl QLinear + SteQuant nvfp4, torch-path quantize, fp32 tables)",
        "optimizer": "torch.optim.AdamW lr 3e-4 betas (0.9, 0.95) wd 0, clip_grad_norm_ 1.0",
        "loss": losses, "grad_norm": gnorms,
    }
    with open(os.path.join(HERE, f"loss_curve_{args.spec}.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
