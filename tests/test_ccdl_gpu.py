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


def test_ccdl_round_matches_reference_golden():
    """Eval-mode round (cdlb200_ccdl_round) against the reference's
    cascaded_nearest_round on the committed cases: codes and scale bytes
    bit-exact, and the eval tensor's dequantize equal to the reference's
    level product for bf16 levels."""
    import os

    from cdl_b200.core.kernel.ccdl import ccdl_round
    from cdl_b200.model.components.quant.ccdl import PackedCcdlTensor

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ccdl_round.npz"))
    names = {E.NVFP4: "nvfp4", E.MXFP4: "mxfp4", E.MXFP8: "mxfp8"}
    for i in range(int(z["count"])):
        c = {k.split("_", 1)[1]: z[k] for k in z.files if k.startswith(f"c{i}_")}
        fmt = int(c["fmt"])
        tpb = 16 if fmt == E.NVFP4 else 32
        dt = torch.bfloat16 if bool(c["theta_bf16"]) else torch.float32
        lt = torch.bfloat16 if bool(c["levels_bf16"]) else torch.float32
        theta = torch.from_numpy(c["theta"]).to(dt).cuda()
        theta = theta.reshape(theta.shape[0], -1, tpb)
        nb = theta.shape[1]
        q = torch.from_numpy(c["q"]).cuda()
        q = q.reshape(1, nb, 1) if q.shape[0] == 1 else q.reshape(-1, nb, 1)
        alpha = torch.tensor(float(c["alpha"]), device="cuda")
        packed, scale = ccdl_round(theta, q, alpha, fmt, lt)
        got_p = packed.view(torch.uint8).reshape(theta.shape[0], -1).cpu().numpy()
        assert np.array_equal(got_p, c["packed"]), f"case {i}: codes"
        assert np.array_equal(scale.cpu().numpy().reshape(c["scale"].shape), c["scale"]), f"case {i}: scales"
        if "deq" in c:
            t = PackedCcdlTensor(names[fmt], packed, scale, alpha, None, nb * tpb, lt, eval_dtype=lt)
            assert np.array_equal(t.dequantize().float().cpu().numpy(), c["deq"]), f"case {i}: dequantize"


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
def test_ccdl_modules_in_a_qlinear(fmt):
    """CCDL activation + weight quantizers in a QLinear under a model with the
    CCDL mixin: the calibration pass sets the activation scales, the
    block-scaled GEMM agrees with dequantize-then-matmul on the same sampled
    codes, gradients reach the input, the weight and every quantizer
    parameter, and eval mode rounds as the oracle does."""
    from torch import nn

    from cdl_b200.core.mm import native
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant import ccdl as Q

    act_cls = {"nvfp4": Q.Nvfp4CascadedCdlQuantForActivation, "mxfp4": Q.Mxfp4CascadedCdlQuantForActivation,
               "mxfp8": Q.Mxfp8CascadedCdlQuantForActivation}[fmt]
    w_cls = {"nvfp4": Q.Nvfp4CascadedCdlQuantForWeight, "mxfp4": Q.Mxfp4CascadedCdlQuantForWeight,
             "mxfp8": Q.Mxfp8CascadedCdlQuantForWeight}[fmt]

    class Model(Q.CascadedCdlQuantMixin):
        def __init__(self):
            super().__init__()
            self.lin = QLinear(256, 128, bias=False, device="cuda", dtype=torch.bfloat16)

        def forward(self, x):
            return self.lin(x)

    torch.manual_seed(0)
    model = Model()
    lin = model.lin
    lin.set_activation_quant(act_cls((1, 256), 5, 5, torch.bfloat16, 2.0).cuda())
    lin.set_weight_quant(w_cls(lin.weight, torch.bfloat16, 2.0).cuda())
    x = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        lin.activation_quant(x)
    # calibration runs on the native backend, as cdl's init_activation_q does
    lin.set_backend("native")
    model.cascaded_cdl_init_act_q_pass([x])
    lin.set_backend(fmt)
    aq = lin.activation_quant
    assert aq.initialized and aq.log_q.shape == (1, 256 // aq.block_size, 1)
    top = 448.0 if fmt == "mxfp8" else 6.0
    bamax = x.float().abs().reshape(64, -1, aq.block_size).amax(-1).amax(0)
    assert torch.allclose(aq.q.reshape(-1), bamax / top, rtol=2e-2)  # q and its log in bf16
    assert model.cascaded_cdl_get_activation_quant_counts() == 256
    assert model.cascaded_cdl_get_weight_quant_counts() == 128 * 256

    x = x.requires_grad_()
    xq, wq = lin.activation_quant(x), lin.weight_quant(lin.weight)
    out = lin.available_backend_fn[fmt](xq, wq)
    ref = native.matmul(xq, wq)
    assert float((out.detach().float() - ref.detach().float()).norm() / ref.detach().float().norm()) < 2e-2
    (out.float() ** 2).sum().backward()
    for m in (lin.activation_quant, lin.weight_quant):
        for p in (m.log_q, m.log_alpha, m.log_theta_kappa, m.log_q_kappa):
            assert p.grad is not None and bool(torch.isfinite(p.grad).all())
    for t in (x, lin.weight):
        assert t.grad is not None and bool(torch.isfinite(t.grad).all())
    assert int(aq.kernel_seed) == 1

    model.eval()
    wq = lin.weight_quant(lin.weight)
    fid = {"nvfp4": E.NVFP4, "mxfp4": E.MXFP4, "mxfp8": E.MXFP8}[fmt]
    tpb = lin.weight_quant.block_size
    op, osc = E.ccdl_round(fid, lin.weight.detach().float().cpu().numpy().reshape(128, -1, tpb),
                           lin.weight_quant.q.detach().cpu().numpy().reshape(128, -1),
                           float(lin.weight_quant.alpha), True, True)
    assert np.array_equal(wq.packed_theta.view(torch.uint8).reshape(128, -1).cpu().numpy(), op)
    assert np.array_equal(wq.packed_scale.reshape(128, -1).cpu().numpy(), osc)
    y = model(x.detach())
    assert y.shape == (64, 128) and bool(torch.isfinite(y.float()).all())
    groups, params = model.cascaded_cdl_get_param_groups(1e-3, train_alpha=True, train_kappa=False)
    assert len(params) == 8 and not lin.weight_quant.log_q_kappa.requires_grad
