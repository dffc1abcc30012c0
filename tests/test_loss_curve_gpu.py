"""Loss-curve parity of the B200 QAT step against the reference's own step,
run twice: on the host cores (a committed fixture, below) and on the same GPU
(``test_loss_curve_matches_reference_step_on_gpu``: the reference's unmodified
step from ``baseline/_ref`` at BASELINE config C4).

``tests/golden/loss_curve_135m.json`` was made by
``tests/golden/make_loss_curve.py``: the reference's QLinear + SteQuant
("nvfp4") + native backend (dequantize, bf16 matmul, STE) on every linear of a
random-init SmolLM2-135M (BASELINE config C4 dimensions), cross entropy
through the unquantized head, clip 1.0 + AdamW (lr 3e-4, betas 0.9/0.95),
run on the CPU from seed 0 for 200 steps on seeded uniform token batches
(smaller than C4's 8 x 2048 tokens per step so that the reference run on the
host cores ends in about half an hour; the fixture records its batch).

Here the same model (drawn on the CPU from the same seed) and the same
batches train on the GPU with the ``nvfp4`` backend (FP4 forward GEMM, bf16
backward: the reference's numerics) and the ``nvfp4_qbwd`` backend (FP4
forward, dgrad and wgrad).  BASELINE criterion: the loss stays within 0.5 %
of the reference's at every one of the 200 steps.  The gradient norms of the
first steps, which move most, are compared too.
"""

import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _reference():
    with open(os.path.join(HERE, "golden", "loss_curve_135m.json")) as f:
        return json.load(f)


def _moving_average(v, w=10):
    return [sum(v[i:i + w]) / w for i in range(len(v) - w + 1)]


@pytest.mark.parametrize("backend,gnorm0_tol", [("nvfp4", 0.03), ("nvfp4_qbwd", 0.10)])
def test_loss_curve_matches_reference_200_steps(backend, gnorm0_tol):
    """Criteria, all against the reference curve:

    * the 10-step moving average of the loss within 0.5 % everywhere -- the
      curve; single steps of uniform-random-token training are noisy, and the
      CPU and GPU runs of the same model drift apart step by step through
      arithmetic differences alone (the ``native`` backend, the reference's
      own numerics on this GPU, reaches 0.45 % on single steps);
    * every single step within 1 %, the 200-step mean within 0.1 %;
    * the first step's gradient norm (same weights, same batch) within
      ``gnorm0_tol`` (the FP4 dgrad / wgrad of ``nvfp4_qbwd`` change the
      gradients themselves).  Later gradient norms are reported, not
      asserted: the fixture's reference ran on the CPU, where cdl's
      ``gmax / 2688`` is a true division, while on the device (and here) it is
      a multiply by the reciprocal, so about a fifth of all tensors get a
      one-ulp different alpha; on noisy random-token training such a
      perturbation moves the gradient-norm spikes of later steps while the
      loss curve stays within the criteria.  The GPU test below compares
      against the reference's step on the device, where the arithmetic is
      the same, under the strict per-step criterion."""
    from cdl_b200 import workloads
    from cdl_b200.train import qat

    ref = _reference()
    assert ref["steps"] >= 200 and len(ref["loss"]) == ref["steps"]
    spec = qat.SPECS[ref["spec"]]
    dev = torch.device("cuda")
    step = qat.QatStep(spec, dev, backend=backend, lr=3e-4, seed=ref["seed"], init_device="cpu")
    losses, gnorms = [], []
    for ids in workloads.token_batches(ref["batch"], ref["seq"], spec.vocab, ref["seed"], ref["steps"]):
        loss, gn = step.step(ids.to(dev))
        losses.append(loss)
        gnorms.append(gn)
    step.check_status()
    losses = [float(v) for v in losses]
    gnorms = [float(v) for v in gnorms]
    rel = [abs(a - b) / b for a, b in zip(losses, ref["loss"])]
    ma = [abs(a - b) / b for a, b in zip(_moving_average(losses), _moving_average(ref["loss"]))]
    mean_rel = abs(sum(losses) - sum(ref["loss"])) / sum(ref["loss"])
    med = sorted(gnorms)[len(gnorms) // 2] / sorted(ref["grad_norm"])[len(gnorms) // 2]
    print(f"{backend}: worst single step {max(rel):.4%}, worst 10-step average {max(ma):.4%}, "
          f"mean {mean_rel:.4%}, first grad norm {gnorms[0]:.4f} vs {ref['grad_norm'][0]:.4f}, "
          f"median grad norm ratio {med:.4f}, mean grad norm ratio {sum(gnorms) / sum(ref['grad_norm']):.4f}")
    assert max(ma) < 5e-3, max(ma)
    assert max(rel) < 1e-2, max(rel)
    assert mean_rel < 1e-3, mean_rel
    assert abs(gnorms[0] - ref["grad_norm"][0]) / ref["grad_norm"][0] < gnorm0_tol


_REF_CURVE = {}


def _reference_curve_gpu(spec_name, batch, seq, steps, seed):
    """Loss and gradient norm per step of the reference's own step
    (``baseline/reference_step.py``: cdl's QLinear + SteQuant("nvfp4") with the
    Triton quantizers, the native backend, Liger's loss, torch AdamW) on this
    GPU; computed once per configuration."""
    import sys

    root = os.path.dirname(HERE)
    if root not in sys.path:
        sys.path.insert(0, root)
    from baseline import reference_step

    reason = reference_step.unavailable()
    if reason is not None:
        pytest.skip(f"reference step unavailable: {reason}")
    key = (spec_name, batch, seq, steps, seed)
    if key not in _REF_CURVE:
        from cdl_b200 import workloads
        from cdl_b200.train import qat

        spec = qat.SPECS[spec_name]
        dev = torch.device("cuda")
        ref = reference_step.ReferenceQatStep(spec, dev, lr=3e-4, seed=seed)
        out = [ref.step(ids.to(dev)) for ids in workloads.token_batches(batch, seq, spec.vocab, seed, steps)]
        _REF_CURVE[key] = ([float(v[0]) for v in out], [float(v[1]) for v in out])
        del ref
        torch.cuda.empty_cache()
    return _REF_CURVE[key]


@pytest.mark.parametrize("backend", ["nvfp4", "nvfp4_qbwd"])
def test_loss_curve_matches_reference_step_on_gpu(backend):
    """BASELINE config C4 (SmolLM2-135M, 8 x 2048 tokens per step), 200 steps
    from seed 0: this library's step against the reference's own step run on
    the same GPU from the same initial weights and batches.  Criterion (the
    north star's): the loss within 0.5 % of the reference's at every step;
    the first step's gradient norm (same weights, same batch) within 1 %
    (``nvfp4``, the reference's numerics) / 10 % (``nvfp4_qbwd``: FP4 dgrad and
    wgrad change the gradients themselves)."""
    from cdl_b200 import workloads
    from cdl_b200.train import qat

    batch, seq, steps, seed = 8, 2048, 200, 0
    ref_loss, ref_gn = _reference_curve_gpu("135m", batch, seq, steps, seed)
    spec = qat.SPECS["135m"]
    dev = torch.device("cuda")
    step = qat.QatStep(spec, dev, backend=backend, lr=3e-4, seed=seed, init_device="cpu")
    out = [step.step(ids.to(dev)) for ids in workloads.token_batches(batch, seq, spec.vocab, seed, steps)]
    step.check_status()
    losses = [float(v[0]) for v in out]
    gnorms = [float(v[1]) for v in out]
    rel = [abs(a - b) / b for a, b in zip(losses, ref_loss)]
    mean_rel = abs(sum(losses) - sum(ref_loss)) / sum(ref_loss)
    med = sorted(gnorms)[steps // 2] / sorted(ref_gn)[steps // 2]
    print(f"{backend} vs reference step on GPU: worst step {max(rel):.4%} (step {rel.index(max(rel))}), "
          f"mean {mean_rel:.4%}, first grad norm {gnorms[0]:.4f} vs {ref_gn[0]:.4f}, "
          f"median grad norm ratio {med:.4f}, mean grad norm ratio {sum(gnorms) / sum(ref_gn):.4f}, "
          f"losses {losses[0]:.4f}->{losses[-1]:.4f} vs {ref_loss[0]:.4f}->{ref_loss[-1]:.4f}")
    assert max(rel) < 5e-3, max(rel)
    tol = 0.01 if backend == "nvfp4" else 0.10
    assert abs(gnorms[0] - ref_gn[0]) / ref_gn[0] < tol
