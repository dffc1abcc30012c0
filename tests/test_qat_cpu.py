"""CPU checks of the QAT step's host-side pieces."""

import torch
import torch.nn.functional as F


def test_linear_cross_entropy_matches_plain_path():
    from cdl_b200.train.qat import LinearCrossEntropy

    torch.manual_seed(0)
    h = torch.randn(300, 64, requires_grad=True)
    w = (0.05 * torch.randn(1000, 64)).requires_grad_()
    t = torch.randint(0, 1000, (300,))
    loss = LinearCrossEntropy.apply(h, w, t, 128)
    (2.0 * loss).backward()
    gh, gw = h.grad.clone(), w.grad.clone()
    h.grad = w.grad = None
    ref = F.cross_entropy(h @ w.t(), t)
    (2.0 * ref).backward()
    assert torch.allclose(loss, ref, rtol=1e-6)
    assert torch.allclose(gh, h.grad, rtol=1e-5, atol=1e-7)
    assert torch.allclose(gw, w.grad, rtol=1e-5, atol=1e-7)


def test_quantized_backward_backend_names():
    from cdl_b200.model.components.linear import QLinear

    q = QLinear(64, 32)
    for be in ("native", "nvfp4", "mxfp4", "mxfp8", "nvfp4_qbwd", "mxfp4_qbwd", "mxfp8_qbwd"):
        q.set_backend(be)
    try:
        q.set_backend("fp4")
    except ValueError:
        pass
    else:
        raise AssertionError("unknown backend accepted")
