"""GPU parity of the CCDL kernels (csrc/ecdl.cu) against the oracle
(oracle/ecdl.py): sampled scale bytes and codes, proxy gradients for theta
and q, the kappa / alpha sums, and the autograd wrapper."""

import numpy as np
import pytest
import torch

from oracle import ecdl as E

pytestmark = pytest.mark.gpu

# (format, block, theta topk, q topk, shared q row)
CASES = [(E.NVFP4, 16, 5, 5, False), (E.NVFP4, 16, 16, 3, True), (E.MXFP4, 32, 6, 5, False),
         (E.MXFP8, 32, 8, 5, False)]


def _inputs(fmt, tpb, shared, seed):
    g = torch.Generator().manual_seed(seed)
    theta = (torch.randn(32, 12, tpb, generator=g) * torch.exp(torch.randn(32, 12, 1, generator=g))).bfloat16()
    bamax = theta.float().abs().amax(-1)
    if fmt == E.NVFP4:
        alpha = float(bamax.max()) / 2688.0
        q = (bamax / (6.0 * alpha)).clamp(0.01, 440.0)
    else:
        alpha = 1.0
        q = (bamax / (4.0 if fmt == E.MXFP4 else 256.0)).clamp_min(1e-6)
    if shared:
        q = q[:1].clone()
    return theta, q.float(), alpha


@pytest.mark.parametrize("fmt,tpb,topk,qtopk,shared", CASES)
def test_ccdl_forward_and_backward_match_oracle(fmt, tpb, topk, qtopk, shared):
    from cdl_b200.core.kernel.ccdl import ccdl_quant_bwd, ccdl_quant_fwd

    theta, q, alpha = _inputs(fmt, tpb, shared, 10 + fmt)
    kt, kq, seed = 3.0, 2.0, 17
    dev = "cuda"
    t = lambda v: torch.tensor(v, dtype=torch.float32, device=dev)  # noqa: E731
    qd = q.reshape(12) if shared else q
    packed, scale = ccdl_quant_fwd(theta.cuda(), qd.cuda(), t(kt), t(kq), t(alpha),
                                   torch.tensor(seed, device=dev), fmt, topk, qtopk)
    op, osc = E.ccdl_forward(fmt, theta.float().numpy(), q.numpy().reshape(-1, 12), kt, kq, alpha, seed, topk, qtopk)
    assert np.array_equal(scale.cpu().numpy().reshape(osc.shape), osc)
    same = float(np.mean(packed.view(torch.uint8).cpu().numpy().reshape(op.shape) == op))
    print(f"fmt {fmt}: codes equal {same:.6f}")
    assert same > 0.999
    g = torch.randn(theta.shape, generator=torch.Generator().manual_seed(3)).bfloat16()
    dth, dq, sc = ccdl_quant_bwd(g.cuda(), theta.cuda(), qd.cuda(), scale, t(kt), t(kq), t(alpha), fmt, topk, qtopk,
                                 True, True, True, True)
    odth, odq, osc3 = E.ccdl_backward(fmt, g.float().numpy(), theta.float().numpy(), q.numpy().reshape(-1, 12),
                                      osc, kt, kq, alpha, topk, qtopk)
    ref = torch.from_numpy(odth).bfloat16().float()
    got = dth.float().cpu().reshape(ref.shape)
    bad = (got - ref).abs() > (2 ** -7 * ref.abs() + 1e-3 * float(ref.abs().max()))
    assert float(bad.float().mean()) < 1e-3
    rq = torch.from_numpy(odq)
    gq = dq.cpu().reshape(rq.shape)
    assert float((gq - rq).norm() / rq.norm().clamp_min(1e-30)) < 1e-3
    for a, b in zip(sc.cpu().tolist(), osc3):
        assert abs(a - b) <= 1e-3 * max(1.0, abs(b)), (a, b)


def test_ccdl_autograd():
    from cdl_b200.core.kernel.ccdl import nvfp4_ccdl_quant

    theta, q, alpha = _inputs(E.NVFP4, 16, False, 5)
    theta = theta.cuda().requires_grad_()
    q = q.cuda().requires_grad_()
    kt = torch.tensor(3.0, device="cuda", requires_grad=True)
    kq = torch.tensor(2.0, device="cuda", requires_grad=True)
    al = torch.tensor(alpha, device="cuda", requires_grad=True)
    seed = torch.zeros((), dtype=torch.int64, device="cuda")
    packed, scale, carrier = nvfp4_ccdl_quant(theta, q, kt, kq, al, seed, 5, 5)
    assert int(seed) == 1 and scale.shape == (32, 12, 1)
    (carrier * torch.randn_like(carrier)).sum().backward()
    for x in (theta, q, kt, kq, al):
        assert x.grad is not None and bool(torch.isfinite(x.grad).all())
    assert q.grad.shape == q.shape
