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
    for be in ("native", "nvfp4", "nvfp4_qbwd"):
        step = qat.QatStep(spec, dev, backend=be, lr=3e-4, seed=0)
        losses, gns = [], []
        for i in range(60):
            ids = qat.random_tokens(8, 256, spec.vocab, seed=100 + i, device=dev)
            loss, gn = step.step(ids)
            losses.append(float(loss))
            gns.append(float(gn))
        curves[be], norms[be] = losses, gns
    assert abs(curves["native"][0] - qat.expected_initial_loss(spec)) < 0.5
    for be in ("nvfp4", "nvfp4_qbwd"):
        for a, b in zip(curves[be], curves["native"]):
            assert abs(a - b) / b < 5e-3, (be, a, b)
    for a, b in zip(norms["nvfp4"][:10], norms["native"][:10]):
        assert abs(a - b) / b < 5e-2, (a, b)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
def test_quantized_backward_gemms_vs_oracle(fmt):
    """dgrad = Q(g).Q(w^T)^T and wgrad = Q(g^T).Q(x^T)^T against the fp32
    dequantize-then-matmul oracle of the same quantized operands."""
    import numpy as np

    import oracle
    from cdl_b200.core.mm.blockscaled import _quantized_grads

    ofmt = {"nvfp4": oracle.NVFP4, "mxfp4": oracle.MXFP4, "mxfp8": oracle.MXFP8}[fmt]
    gen = torch.Generator("cuda").manual_seed(5)
    m, n, k = 256, 320, 576
    g = torch.randn(m, n, device="cuda", generator=gen).bfloat16()
    x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    w = (0.02 * torch.randn(n, k, device="cuda", generator=gen)).bfloat16()
    dx, dw = _quantized_grads(fmt, g, x, w)
    assert dx.shape == (m, k) and dw.shape == (n, k)

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    def qmm(a, b):  # oracle of alpha * deq(Q(a)) @ deq(Q(b))^T, both quantized along their rows
        ap, asf, aal = oracle.quant(bits(a), ofmt)
        bp, bsf, bal = oracle.quant(bits(b), ofmt)
        alpha = 1.0 if aal is None else float(aal[0]) * float(bal[0])
        return oracle.mm(ap, asf, bp, bsf, ofmt, alpha)

    for got, ref in ((dx, qmm(g, w.t())), (dw, qmm(g.t(), x.t()))):
        ref_bf16 = torch.from_numpy(ref).bfloat16().float()
        assert _rel(got.cpu(), ref_bf16) <= 1e-3


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp8"])
def test_qlinear_quantized_backward_close_to_reference_grads(fmt):
    """The *_qbwd backends' gradients stay within the quantization error of
    the reference (bf16) backward."""
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant.ste import SteQuant

    torch.manual_seed(0)
    lin = torch.nn.Linear(576, 320, bias=False).cuda().bfloat16()
    grads = {}
    for be in (fmt, fmt + "_qbwd"):
        q = QLinear.from_linear(lin)
        q.set_activation_quant(SteQuant(fmt))
        q.set_weight_quant(SteQuant(fmt))
        q.set_backend(be)
        x = torch.randn(3, 128, 576, device="cuda", dtype=torch.bfloat16, generator=torch.Generator("cuda").manual_seed(1))
        x.requires_grad_(True)
        y = q(x)
        y.backward(torch.randn_like(y, generator=torch.Generator("cuda").manual_seed(2)))
        grads[be] = (x.grad.detach(), q.weight.grad.detach())
    bound = 0.25 if fmt == "nvfp4" else 0.08
    for a, b in zip(grads[fmt + "_qbwd"], grads[fmt]):
        assert _rel(a, b) < bound, _rel(a, b)


def test_loss_curve_quantized_backward():
    """NVFP4 fwd/dgrad/wgrad (nvfp4_qbwd) against NVFP4 fwd + bf16 backward
    (cdl's numerics): same seed and data, 60 steps on the small model."""
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    curves = {}
    for be in ("nvfp4", "nvfp4_qbwd"):
        step = qat.QatStep(spec, dev, backend=be, lr=3e-4, seed=0)
        curves[be] = [float(step.step(qat.random_tokens(8, 256, spec.vocab, seed=100 + i, device=dev))[0])
                      for i in range(60)]
    worst = max(abs(a - b) / b for a, b in zip(curves["nvfp4_qbwd"], curves["nvfp4"]))
    print("max relative loss difference, quantized vs bf16 backward:", worst)
    assert worst < 2e-2



def test_graph_step_matches_eager():
    """The CUDA-graph step (three warm-up steps and the capture on the first
    batch, then replays with fresh tokens copied into the static input) follows
    the loss curve of the eager step on the same sequence of batches."""
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    batches = [qat.random_tokens(8, 256, spec.vocab, seed=200 + i, device=dev) for i in range(12)]
    graph = qat.QatStep(spec, dev, backend="nvfp4", lr=3e-4, seed=0, graph=True)
    got = [float(graph.step(b)[0]) for b in batches]
    eager = qat.QatStep(spec, dev, backend="nvfp4", lr=3e-4, seed=0)
    for _ in range(3):
        eager.step(batches[0])
    ref = [float(eager.step(b)[0]) for b in batches]
    print("graph:", got[:4], "eager:", ref[:4])
    worst = max(abs(a - b) / b for a, b in zip(got, ref))
    assert worst < 5e-3


def test_dgrad_sum_in_gemm_epilogue_is_bit_exact():
    """The quantized backward adds the input gradients of the linears that
    share an input (q / k / v, gate / up) in the dgrad GEMMs' epilogue
    instead of leaving the sums to autograd's adds; the step's losses,
    gradient norms and parameters are the same bits either way."""
    from cdl_b200.core.mm import blockscaled
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    batches = [qat.random_tokens(4, 256, spec.vocab, seed=300 + i, device=dev) for i in range(3)]
    runs = []
    try:
        for fuse in (True, False):
            blockscaled.FUSE_DGRAD_SUM = fuse
            step = qat.QatStep(spec, dev, backend="nvfp4_qbwd", lr=1e-3, seed=0)
            n0 = blockscaled.dgrad_accumulates
            out = [tuple(float(v) for v in step.step(b)) for b in batches]
            # per layer and step: k and v add into q's dgrad, up into gate's
            assert blockscaled.dgrad_accumulates - n0 == (3 * spec.layers * len(batches) if fuse else 0)
            flat = torch.cat([p.detach().reshape(-1).view(torch.int16) for p in step.model.parameters()])
            runs.append((out, flat))
    finally:
        blockscaled.FUSE_DGRAD_SUM = True
    assert runs[0][0] == runs[1][0]
    assert torch.equal(runs[0][1], runs[1][1])


@pytest.mark.parametrize("activation,weight", [("ste", "nvfp4_ccdl"), ("nvfp4_ccdl", "nvfp4_ccdl"),
                                               ("nvfp4_ecdl", "nvfp4_ecdl")])
def test_qat_step_with_cdl_quantizers(activation, weight):
    """The QAT step with cdl's CDL quantizer variants (its default config is
    CCDL weights with STE activations): CCDL activations are calibrated on the
    native backend first; the loss starts near log(vocab), stays finite and
    falls; the quantizer parameters move."""
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    step = qat.QatStep(spec, dev, backend="nvfp4", lr=1e-3, seed=0, activation=activation, weight=weight,
                       train_kappa=True)  # ECDL's only parameter is its temperature
    if activation.endswith("ccdl"):
        step.calibrate([qat.random_tokens(2, 128, spec.vocab, seed=7, device=dev)])
    wq = next(m for m in step.model.modules() if isinstance(m, QLinear)).weight_quant
    before = [p.detach().clone() for p in wq.parameters() if p.requires_grad]
    losses = []
    for i in range(12):
        ids = qat.random_tokens(4, 128, spec.vocab, seed=i % 3, device=dev)
        loss, gn = step.step(ids)
        losses.append(float(loss))
        assert torch.isfinite(gn)
    assert abs(losses[0] - qat.expected_initial_loss(spec)) < 0.5
    assert all(map(lambda v: v == v and abs(v) < 1e3, losses)) and min(losses[-3:]) < losses[0]
    after = [p.detach() for p in wq.parameters() if p.requires_grad]
    assert before and any(not torch.equal(a, b) for a, b in zip(before, after))


def test_qat_step_lora_with_warmup():
    """cdl's default regime: LoRA adapters on every quantized linear, base
    weights and head frozen, warmup schedule; the adapters move, the base
    weights do not, and the loss falls."""
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    step = qat.QatStep(spec, dev, backend="nvfp4", lr=3e-3, seed=0, use_lora=True, warmup_steps=3)
    assert step.optimizer == "fused"
    lin = next(m for m in step.model.modules() if isinstance(m, QLinear))
    w0, b0 = lin.weight.detach().clone(), lin.lora.b.detach().clone()
    losses = []
    for i in range(10):
        loss, gn = step.step(qat.random_tokens(4, 128, spec.vocab, seed=i % 2, device=dev))
        losses.append(float(loss))
        assert torch.isfinite(gn)
    assert step.opt.param_groups[0]["lr"] == pytest.approx(3e-3)
    assert torch.equal(lin.weight.detach(), w0) and not torch.equal(lin.lora.b.detach(), b0)
    assert min(losses[-3:]) < losses[0]


def test_dual_quantized_backward_matches_oracle_checked_path():
    """The nvfp4_qbwd QLinear with every dimension a multiple of 64 runs on
    the dual encodings (x, w in the forward, g in the backward); its output
    and gradients equal, bit for bit, the nvfp4 forward and the quantized
    gradients of the single-direction path checked against the oracle above."""
    from cdl_b200.core.mm.blockscaled import _quantized_grads
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant.ste import SteQuant

    torch.manual_seed(0)
    lin = torch.nn.Linear(576, 320, bias=False).cuda().bfloat16()
    res = {}
    for be in ("nvfp4", "nvfp4_qbwd"):
        q = QLinear.from_linear(lin)
        q.set_activation_quant(SteQuant("nvfp4"))
        q.set_weight_quant(SteQuant("nvfp4"))
        q.set_backend(be)
        x = torch.randn(3, 128, 576, device="cuda", dtype=torch.bfloat16,
                        generator=torch.Generator("cuda").manual_seed(1)).requires_grad_(True)
        y = q(x)
        g = torch.randn_like(y, generator=torch.Generator("cuda").manual_seed(2))
        y.backward(g)
        res[be] = (y.detach(), x.grad.detach(), q.weight.grad.detach(), x.detach(), g)
    assert torch.equal(res["nvfp4"][0], res["nvfp4_qbwd"][0])
    y, dx, dw, x, g = res["nvfp4_qbwd"]
    rdx, rdw = _quantized_grads("nvfp4", g.reshape(-1, 320).contiguous(), x.reshape(-1, 576), lin.weight.detach())
    assert torch.equal(dx.reshape(-1, 576), rdx)
    assert torch.equal(dw, rdw)


def test_optimizer_dual_weight_encodings():
    """After a step of the nvfp4_qbwd QAT step, every weight carries the
    optimizer's encodings of w and w^T, equal to the quantizers' own."""
    from cdl_b200.core.kernel.quant import nvfp4_quant
    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.train import qat
    from cdl_b200.train.optim import ENCODED_ATTR

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    step = qat.QatStep(spec, dev, backend="nvfp4_qbwd", seed=0)
    step.step(qat.random_tokens(2, 128, spec.vocab, seed=0, device=dev))
    qls = [m for m in step.model.modules() if isinstance(m, QLinear)]
    assert qls
    for m in qls:
        enc = getattr(m.weight, ENCODED_ATTR)
        assert enc[0] == m.weight._version and enc[4] is None
        p, s, a = nvfp4_quant(m.weight.detach(), swizzled=True)
        tp, ts, _ = nvfp4_quant(m.weight.detach(), transpose=True, swizzled=True)
        assert torch.equal(enc[1], p) and torch.equal(enc[2], s) and torch.equal(enc[3], a)
        assert torch.equal(enc[5], tp) and torch.equal(enc[6], ts)
