"""ClipAdamW (cdlb200_clip_adamw) against torch's clip_grad_norm_ +
AdamW(fused=True) on bf16 tensors, the pair the reference's step runs."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SIZES = [8, 24, 2048, 16384, 16392, 100000, 256 * 1024, 2048 * 2048 + 8]


def _ulp_diff(a, b):
    """|a - b| in units of the bf16 spacing at max(|a|, |b|)."""
    a, b = a.float(), b.float()
    mag = torch.maximum(a.abs(), b.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    return ((a - b).abs() / ulp)


@pytest.mark.parametrize("weight_decay", [0.0, 0.1])
@pytest.mark.parametrize("grad_scale", [1e-4, 1.0])  # clip inactive / active
def test_clip_adamw_matches_torch(grad_scale, weight_decay):
    """Bit-level parity with the reference's optimizer: clip_grad_norm_
    (foreach) then torch.optim.AdamW with its default foreach implementation
    (what cdl's training script constructs), on bf16 tensors over four steps."""
    from cdl_b200.train.optim import ClipAdamW

    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    init = [(torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16) for n in SIZES]
    ours = [t.clone().requires_grad_() for t in init]
    ref = [t.clone().requires_grad_() for t in init]
    opt = ClipAdamW(ours, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=weight_decay, max_norm=1.0)
    topt = torch.optim.AdamW(ref, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=weight_decay, foreach=True)
    for step in range(4):
        grads = [(torch.randn(n, device=dev, generator=gen) * grad_scale).to(torch.bfloat16) for n in SIZES]
        for p, q, g in zip(ours, ref, grads):
            p.grad, q.grad = g.clone(), g.clone()
        norm = opt.step()
        tnorm = torch.nn.utils.clip_grad_norm_(ref, 1.0, foreach=True)
        topt.step()
        opt.zero_grad()
        topt.zero_grad()
        assert abs(float(norm) - float(tnorm)) <= float(tnorm) * 2 ** -7, (step, float(norm), float(tnorm))
        for name, mine, theirs in (("param", ours, ref),
                                   ("exp_avg", opt.exp_avg, [topt.state[q]["exp_avg"] for q in ref]),
                                   ("exp_avg_sq", opt.exp_avg_sq, [topt.state[q]["exp_avg_sq"] for q in ref])):
            a = torch.cat([x.detach().reshape(-1) for x in mine])
            b = torch.cat([x.detach().reshape(-1) for x in theirs])
            frac = float((a != b).float().mean())
            d = _ulp_diff(a, b)
            print(step, name, "elements differing", frac, "max ulp", float(d.max()))
            # identical up to the last bit of a host-side scalar (pow / sqrt
            # of the bias corrections), which moves a handful of roundings
            assert frac < 1e-4, (step, name)
            assert float(d.max()) <= 1.0, (step, name)
    assert opt.steps_done == 4


def test_clip_adamw_deterministic_and_capturable():
    """Two runs give identical bits; the same step captured in a CUDA graph
    and replayed gives identical bits too."""
    from cdl_b200.train.optim import ClipAdamW

    dev = torch.device("cuda")

    def run(graph):
        gen = torch.Generator(device=dev).manual_seed(1)
        ps = [(torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16).requires_grad_() for n in SIZES]
        gs = [torch.randn(n, device=dev, generator=gen).to(torch.bfloat16) for n in SIZES]
        opt = ClipAdamW(ps, lr=1e-3, betas=(0.9, 0.95), max_norm=1.0)
        for p, g in zip(ps, gs):
            p.grad = g
        if graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                opt.step()
            torch.cuda.current_stream().wait_stream(s)
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg):
                out = opt.step()
            for _ in range(3):
                cg.replay()
        else:
            for _ in range(4):
                out = opt.step()
        torch.cuda.synchronize()
        return [p.detach().clone() for p in ps], float(out)

    a, na = run(False)
    b, nb = run(False)
    c, nc = run(True)
    assert na == nb == nc
    for x, y, z in zip(a, b, c):
        assert torch.equal(x, y) and torch.equal(x, z)


def test_qat_step_fused_optimizer_vs_torch():
    """The QAT step with ClipAdamW follows the loss curve of the step with
    torch's clip + AdamW."""
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    curves = {}
    for optimizer in ("fused", "torch"):
        step = qat.QatStep(spec, dev, backend="nvfp4", lr=3e-4, seed=0, optimizer=optimizer)
        curves[optimizer] = [float(step.step(qat.random_tokens(8, 256, spec.vocab, seed=300 + i, device=dev))[0])
                             for i in range(20)]
    worst = max(abs(a - b) / b for a, b in zip(curves["fused"], curves["torch"]))
    print("max relative loss difference, fused vs torch optimizer:", worst)
    assert worst < 5e-3


def _amax_bits(x):
    return int((x.view(torch.int16).int() & 0x7FFF).max())


def test_encode_multi_matches_per_tensor_quantize():
    """cdlb200_nvfp4_encode_multi (amax given) against the per-tensor NVFP4
    quantizer with swizzled scales, and its dequantized copy against the
    dequantizer: bit-identical, for several shapes in one launch."""
    import ctypes

    from cdl_b200 import _lib
    from cdl_b200.core.kernel.dequant import nvfp4_dequant
    from cdl_b200.core.kernel.quant import nvfp4_quant

    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(5)
    shapes = [(128, 64), (256, 512), (2048, 2048), (384, 1088)]
    xs = [(torch.randn(r, k, device=dev, generator=gen) * (0.01 + i)).bfloat16() for i, (r, k) in enumerate(shapes)]
    xs[1][3, 7] = 0.0
    amax = torch.tensor([_amax_bits(x) for x in xs], dtype=torch.int32, device=dev)
    tab = (_lib.Nvfp4EncodeTensor * len(xs))()
    outs = []
    for i, x in enumerate(xs):
        r, k = x.shape
        o = (torch.empty(r, k // 2, dtype=torch.uint8, device=dev), torch.empty(r, k // 16, dtype=torch.uint8, device=dev),
             torch.empty(1, device=dev), torch.empty(r, k, dtype=torch.bfloat16, device=dev))
        outs.append(o)
        t = tab[i]
        t.x, t.rows, t.k, t.amax, t.amax_words = x.data_ptr(), r, k, amax.data_ptr() + 4 * i, 1
        t.packed, t.scale, t.alpha, t.deq = (v.data_ptr() for v in o)
    _lib.call("cdlb200_nvfp4_encode_multi", ctypes.addressof(tab), len(xs), _lib.stream(dev))
    for x, (p, s, a, d) in zip(xs, outs):
        rp, rs, ra = nvfp4_quant(x, swizzled=True)
        assert torch.equal(p, rp) and torch.equal(s, rs) and torch.equal(a.reshape(-1), ra.reshape(-1))
        assert torch.equal(d, nvfp4_dequant(rp, rs, ra, swizzled=True))


def test_optimizer_weight_encoding_is_current():
    """After ClipAdamW.step the encoded weights equal a fresh quantize of the
    updated weights, and a weight modified afterwards falls back (its version
    moved on)."""
    from cdl_b200.core.kernel.quant import nvfp4_quant
    from cdl_b200.train.optim import ENCODED_ATTR, ClipAdamW

    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(6)
    ws = [(torch.randn(r, k, device=dev, generator=gen) * 0.02).bfloat16().requires_grad_()
          for r, k in [(256, 256), (512, 128), (128, 1024)]]
    bias = torch.zeros(64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    opt = ClipAdamW(ws + [bias], lr=1e-2, betas=(0.9, 0.95), encode=ws)
    for step in range(3):
        for w in ws + [bias]:
            w.grad = torch.randn(w.shape, device=dev, generator=gen).bfloat16()
        opt.step()
        opt.zero_grad()
        for w in ws:
            ver, p, s, a, d = getattr(w, ENCODED_ATTR)
            assert ver == w._version
            rp, rs, ra = nvfp4_quant(w.detach(), swizzled=True)
            assert torch.equal(p, rp) and torch.equal(s, rs) and torch.equal(a.reshape(-1), ra.reshape(-1))
    with torch.no_grad():
        ws[0].mul_(2)
    assert getattr(ws[0], ENCODED_ATTR)[0] != ws[0]._version


def test_clip_adamw_state_dict_scheduler_and_torch_checkpoints():
    """ClipAdamW is a torch Optimizer: a LambdaLR schedule drives its lr; its
    state_dict has AdamW's layout; a run resumed from it continues bit for
    bit; and a torch AdamW checkpoint loads into it (and back)."""
    from cdl_b200.train.optim import ClipAdamW

    dev = torch.device("cuda")
    sizes = SIZES[:5]

    def make(seed):
        gen = torch.Generator(device=dev).manual_seed(seed)
        return [(torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16).requires_grad_() for n in sizes]

    def grads(step):
        gen = torch.Generator(device=dev).manual_seed(100 + step)
        return [torch.randn(n, device=dev, generator=gen).to(torch.bfloat16) for n in sizes]

    def run(opt, ps, sched, steps):
        for s in steps:
            for p, g in zip(ps, grads(s)):
                p.grad = g
            opt.step()
            sched.step()
            opt.zero_grad()

    lam = lambda s: min(1.0, (s + 1) / 4)  # noqa: E731
    ps = make(0)
    opt = ClipAdamW(ps, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lam)
    run(opt, ps, sched, range(3))
    assert opt.lr == pytest.approx(1e-3 * 1.0) and opt.param_groups[0]["lr"] == opt.lr
    sd = opt.state_dict()
    assert set(sd["state"][0]) == {"step", "exp_avg", "exp_avg_sq"} and float(sd["state"][0]["step"]) == 3.0
    sd = {"state": {k: {n: t.clone() for n, t in v.items()} for k, v in sd["state"].items()},
          "param_groups": [dict(g) for g in sd["param_groups"]]}
    ssd = sched.state_dict()
    saved = [p.detach().clone() for p in ps]
    run(opt, ps, sched, range(3, 5))
    want = [p.detach().clone() for p in ps]

    # resume: fresh optimizer + scheduler on the saved parameters
    ps2 = [t.clone().requires_grad_() for t in saved]
    opt2 = ClipAdamW(ps2, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
    sched2 = torch.optim.lr_scheduler.LambdaLR(opt2, lam)
    opt2.load_state_dict(sd)
    sched2.load_state_dict(ssd)
    assert opt2.steps_done == 3
    run(opt2, ps2, sched2, range(3, 5))
    for a, b in zip(want, ps2):
        assert torch.equal(a, b.detach())

    # torch AdamW loads our state and continues as our optimizer does
    ref = [t.clone().requires_grad_() for t in saved]
    topt = torch.optim.AdamW(ref, lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, foreach=True)
    tsched = torch.optim.lr_scheduler.LambdaLR(topt, lam)
    topt.load_state_dict(sd)
    tsched.load_state_dict(ssd)
    for s in range(3, 5):
        for p, g in zip(ref, grads(s)):
            p.grad = g
        torch.nn.utils.clip_grad_norm_(ref, 1.0, foreach=True)
        topt.step()
        tsched.step()
        topt.zero_grad()
    a = torch.cat([x.detach().reshape(-1) for x in want])
    b = torch.cat([x.detach().reshape(-1) for x in ref])
    assert float((a != b).float().mean()) < 1e-4 and float(_ulp_diff(a, b).max()) <= 1.0
    # and its state_dict loads into ours
    opt3 = ClipAdamW([t.clone().requires_grad_() for t in want], lr=1e-3)
    opt3.load_state_dict(topt.state_dict())
    assert opt3.steps_done == 5
    assert torch.equal(opt3.exp_avg[2], topt.state[ref[2]]["exp_avg"])
