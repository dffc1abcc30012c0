"""GPU checks of the QAT path: QLinear backends, STE gradients, loss curves."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


@pytest.mark.parametrize("backend", ["nvfp4", "mxfp4", "mxfp8"])
def test_qlinear_backend_matches_native(backend):
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant.ste import SteQuant

    torch.manual_seed(0)
    sim = backend if backend.startswith("mx") else "nvfp4"
    lin = torch.nn.Linear(576, 320, bias=False).cuda().bfloat16()
    outs, grads = {}, {}
    for be in ("native", backend):
        q = QLinear.from_linear(lin)
        q.set_activation_quant(SteQuant(sim))
        q.set_weight_quant(SteQuant(sim))
        q.set_backend(be)
        x = torch.randn(3, 100, 576, device="cuda", dtype=torch.bfloat16, generator=torch.Generator("cuda").manual_seed(1))
        x.requires_grad_(True)
        y = q(x)
        g = torch.randn_like(y, generator=torch.Generator("cuda").manual_seed(2))
        y.backward(g)
        outs[be], grads[be] = y.detach(), (x.grad.detach(), q.weight.grad.detach())
    assert outs[backend].shape == (3, 100, 320)
    # forward: exact FP4 products in fp32 vs bf16-rounded dequantized operands
    assert _rel(outs[backend], outs["native"]) < 1e-2
    # backward: both are g @ deq(W) and g^T @ deq(X) in bf16 (straight-through)
    assert _rel(grads[backend][0], grads["native"][0]) < 1e-2
    assert _rel(grads[backend][1], grads["native"][1]) < 1e-2


def test_loss_curve_nvfp4_vs_native():
    """BASELINE criterion: same seed, uniform random tokens, AdamW lr 3e-4 --
    the NVFP4-GEMM backend's loss curve stays within 0.5% of the
    dequantize-then-matmul (cdl "native") curve at every step."""
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    curves, norms = {}, {}
    for be in ("native", "nvfp4"):
        step = qat.QatStep(spec, dev, backend=be, lr=3e-4, seed=0)
        losses, gns = [], []
        for i in range(60):
            ids = qat.random_tokens(8, 256, spec.vocab, seed=100 + i, device=dev)
            loss, gn = step.step(ids)
            losses.append(float(loss))
            gns.append(float(gn))
        curves[be], norms[be] = losses, gns
    assert abs(curves["native"][0] - qat.expected_initial_loss(spec)) < 0.5
    for a, b in zip(curves["nvfp4"], curves["native"]):
        assert abs(a - b) / b < 5e-3, (a, b)
    for a, b in zip(norms["nvfp4"][:10], norms["native"][:10]):
        assert abs(a - b) / b < 5e-2, (a, b)
