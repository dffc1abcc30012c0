"""GPU parity of the ECDL kernels (csrc/ecdl.cu) against the oracle
(oracle/ecdl.py): scales and alpha exact, sampled codes equal except within
float rounding of a cumulative boundary, proxy gradients and d(kappa) /
d(alpha) to float tolerance; plus the autograd wrapper."""

import numpy as np
import pytest
import torch

from oracle import ecdl as E

pytestmark = pytest.mark.gpu

CASES = [(E.NVFP4, "nvidia", 16, 4), (E.NVFP4, "nvidia", 16, 16), (E.MXFP4, "ocp", 32, 6), (E.MXFP8, "ocp", 32, 8)]


def _theta(m, nb, tpb, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, nb, tpb, generator=g) * torch.exp(torch.randn(m, nb, 1, generator=g))
    x[0, 0] = 0.0  # an all-zero block
    return x.bfloat16()


@pytest.mark.parametrize("fmt,mode,tpb,topk", CASES)
def test_ecdl_forward_matches_oracle(fmt, mode, tpb, topk):
    from cdl_b200.core.kernel.ecdl import ecdl_quant_fwd

    theta = _theta(64, 24, tpb, fmt * 10 + topk)
    kappa, seed = 3.0, 41
    packed, scale, alpha = ecdl_quant_fwd(theta.cuda(), torch.tensor(kappa, device="cuda"),
                                          torch.tensor(seed, dtype=torch.int64, device="cuda"), fmt, topk, mode)
    op, osc, oa, oidx = E.forward(fmt, theta.float().numpy(), kappa, seed, topk,
                                  E.MODE_NVIDIA if mode == "nvidia" else E.MODE_OCP)
    assert np.array_equal(scale.cpu().numpy().reshape(osc.shape), osc)
    assert float(alpha) == float(oa)
    got = packed.view(torch.uint8).cpu().numpy().reshape(op.shape)
    same = float(np.mean(got == op))
    print(f"fmt {fmt} topk {topk}: packed bytes equal {same:.6f}")
    assert same > 0.999


@pytest.mark.parametrize("fmt,mode,tpb,topk", CASES)
def test_ecdl_backward_matches_oracle(fmt, mode, tpb, topk):
    from cdl_b200.core.kernel.ecdl import ecdl_quant_bwd, ecdl_quant_fwd

    theta = _theta(32, 16, tpb, 100 + fmt * 10 + topk)
    kappa = torch.tensor(2.5, device="cuda")
    _, scale, alpha = ecdl_quant_fwd(theta.cuda(), kappa, torch.tensor(5, device="cuda"), fmt, topk, mode)
    g = torch.randn(theta.shape, generator=torch.Generator().manual_seed(9)).bfloat16()
    dth, scalars = ecdl_quant_bwd(g.cuda(), theta.cuda(), scale, kappa, alpha, fmt, topk, mode, True)
    odth, (odk, oda) = E.backward(fmt, g.float().numpy(), theta.float().numpy(),
                                  scale.cpu().numpy().reshape(theta.shape[:2]), 2.5, float(alpha), topk)
    ref = torch.from_numpy(odth).bfloat16().float()
    got = dth.float().cpu().reshape(ref.shape)
    # float32 sums of the window in another order: where the coefficient
    # cancels to near zero the relative error grows, so bound it by the
    # tensor's scale there
    bad = (got - ref).abs() > (2 ** -7 * ref.abs() + 1e-3 * float(ref.abs().max()))
    assert float(bad.float().mean()) < 1e-3, float(bad.float().mean())
    assert abs(float(scalars[0]) - odk) <= 1e-3 * max(1.0, abs(odk))
    assert abs(float(scalars[1]) - oda) <= 1e-3 * max(1.0, abs(oda))


def test_ecdl_sampling_distribution():
    """One value repeated: the sampled levels follow the CDL probabilities."""
    from cdl_b200.core.kernel.ecdl import ecdl_quant_fwd

    n = 1 << 18
    theta = torch.full((n // 16, 1, 16), 1.3, dtype=torch.bfloat16)
    theta[:, :, 0] = 6.0  # block amax 6: s = 1 * alpha with alpha = gmax / 2688 -> v = x / s
    packed, scale, alpha = ecdl_quant_fwd(theta.cuda(), torch.tensor(1.5, device="cuda"),
                                          torch.tensor(77, device="cuda"), E.NVFP4, 8, "nvidia")
    codes = packed.cpu().numpy().reshape(n // 16, 8)
    lo = (codes & 15)[:, 1:]  # elements 2, 4, ... (element 0 is the amax element)
    hi = codes >> 4
    c = np.concatenate([lo.reshape(-1), hi.reshape(-1)])
    f = E.Format(E.NVFP4)
    idx = np.where(c >= 8, 15 - c, c + 8)  # code -> level index
    s = np.float32(E.e4m3_value(np.array([int(scale[0, 0, 0])]))[0] * np.float32(float(alpha)))
    v = np.float32(np.float32(torch.tensor(1.3).bfloat16().float().item()) / s)
    start, p = E.probabilities(f, np.array([v], dtype=np.float32), 1.5, 8)
    freq = np.bincount(idx - start[0], minlength=8)[:8] / idx.size
    assert np.max(np.abs(freq - p[0])) < 5 * np.sqrt(0.25 / idx.size) + 1e-4, (freq, p[0])


def test_ecdl_autograd_seed_and_gradients():
    from cdl_b200.core.kernel.ecdl import ecdl_quant_bwd, nvfp4_ecdl_quant

    theta = _theta(16, 8, 16, 3).cuda().requires_grad_()
    log_kappa = torch.tensor(1.0, device="cuda", requires_grad=True)
    seed = torch.zeros((), dtype=torch.int64, device="cuda")
    packed, scale, carrier, alpha = nvfp4_ecdl_quant(theta, log_kappa.exp(), None, seed, 16)
    assert int(seed) == 1 and not alpha.requires_grad
    g = torch.randn(theta.shape, device="cuda").bfloat16()
    (carrier * g).sum().backward()
    dth, scalars = ecdl_quant_bwd(g, theta.detach(), scale, log_kappa.exp().detach(), alpha, 0, 16, "nvidia", True)
    assert torch.equal(theta.grad.reshape(-1), dth.reshape(-1))
    assert torch.allclose(log_kappa.grad, scalars[0] * log_kappa.exp().detach(), rtol=1e-5)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
def test_ecdl_modules_in_a_qlinear(fmt):
    """ECDL activation + weight quantizers in a QLinear: the block-scaled GEMM
    agrees with dequantize-then-matmul on the same sampled codes, gradients
    reach the input, the weight and both log_kappa, and eval mode rounds."""
    from cdl_b200.core.mm import native
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant import ecdl as Q

    torch.manual_seed(0)
    lin = QLinear(256, 128, bias=False, device="cuda", dtype=torch.bfloat16)
    act_cls = {"nvfp4": Q.Nvfp4ExtendedCdlQuantForActivation, "mxfp4": Q.Mxfp4ExtendedCdlQuantForActivation,
               "mxfp8": Q.Mxfp8ExtendedCdlQuantForActivation}[fmt]
    w_cls = {"nvfp4": Q.Nvfp4ExtendedCdlQuantForWeight, "mxfp4": Q.Mxfp4ExtendedCdlQuantForWeight,
             "mxfp8": Q.Mxfp8ExtendedCdlQuantForWeight}[fmt]
    lin.set_activation_quant(act_cls((1, 256), 5, torch.bfloat16, 4.0).cuda())
    lin.set_weight_quant(w_cls(lin.weight, torch.bfloat16, 4.0).cuda())
    lin.set_backend(fmt)
    x = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    xq, wq = lin.activation_quant(x), lin.weight_quant(lin.weight)
    out = lin.available_backend_fn[fmt](xq, wq)
    ref = native.matmul(xq, wq)
    assert float((out.detach().float() - ref.detach().float()).norm() / ref.detach().float().norm()) < 2e-2
    (out.float() ** 2).sum().backward()
    for t in (x, lin.weight, lin.activation_quant.log_kappa, lin.weight_quant.log_kappa):
        assert t.grad is not None and bool(torch.isfinite(t.grad).all())
    assert int(lin.activation_quant.kernel_seed) == 1
    lin.eval()
    y = lin(x.detach())
    assert y.shape == (64, 128) and bool(torch.isfinite(y.float()).all())
