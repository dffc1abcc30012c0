"""GPU checks of the fused RMSNorm / rotary / SwiGLU kernels against the eager
transformers Llama modules they replace, and of the QAT step with them."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def _max_ulp(a, b):
    """Largest distance in bf16 representable steps between two bf16 tensors."""
    ia = a.contiguous().view(torch.int16).int()
    ib = b.contiguous().view(torch.int16).int()
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return int((ia - ib).abs().max())


@pytest.mark.parametrize("rows,d", [(1000, 576), (300, 2048), (7, 64)])
def test_rmsnorm_matches_eager(rows, d):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    from cdl_b200.model.components.fused import RMSNormFn

    gen = torch.Generator("cuda").manual_seed(rows + d)
    norm = LlamaRMSNorm(d, eps=1e-5).cuda().bfloat16()
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(d, device="cuda", generator=gen))
    x = (3.0 * torch.randn(2, rows, d, device="cuda", generator=gen)).bfloat16()
    g = torch.randn(2, rows, d, device="cuda", generator=gen).bfloat16()
    outs = []
    for fused in (False, True):
        xx = x.clone().requires_grad_(True)
        norm.weight.grad = None
        y = RMSNormFn.apply(xx, norm.weight, 1e-5) if fused else norm(xx)
        y.backward(g)
        outs.append((y.detach(), xx.grad.detach(), norm.weight.grad.detach().clone()))
    (y0, dx0, dw0), (y1, dx1, dw1) = outs
    # the fp32 row sum runs in another order: bf16(x * rstd) may move by one step,
    # which the bf16 product with w can turn into two; such elements are rare
    assert _max_ulp(y1, y0) <= 2
    assert float((y1 != y0).float().mean()) < 0.02
    assert _rel(dx1, dx0) < 1e-2
    assert _rel(dw1, dw0) < 1e-2


def test_rope_matches_eager():
    from transformers.models.llama import modeling_llama as ml

    from cdl_b200.model.components.fused import RopeFn

    gen = torch.Generator("cuda").manual_seed(3)
    b, h, s, d = 2, 4, 96, 64
    cfg = ml.LlamaConfig(hidden_size=h * d, num_attention_heads=h, rope_theta=10000.0, max_position_embeddings=256)
    rot = ml.LlamaRotaryEmbedding(cfg).cuda()
    q0 = torch.randn(b, s, h, d, device="cuda", generator=gen).bfloat16().transpose(1, 2)
    pos = torch.arange(s, device="cuda")[None]
    cos, sin = rot(q0, pos)
    g = torch.randn(b, h, s, d, device="cuda", generator=gen).bfloat16()
    res = []
    for fused in (False, True):
        q = q0.detach().clone().requires_grad_(True)
        if fused:
            out = RopeFn.apply(q, cos, sin)
        else:
            c, sn = cos.unsqueeze(1), sin.unsqueeze(1)
            out = q * c + ml.rotate_half(q) * sn
        out.backward(g)
        res.append((out.detach(), q.grad.detach()))
    assert _max_ulp(res[1][0], res[0][0]) == 0
    assert _max_ulp(res[1][1], res[0][1]) == 0


def test_swiglu_matches_eager():
    from cdl_b200.model.components.fused import SwiGLUFn

    gen = torch.Generator("cuda").manual_seed(4)
    g0 = (2 * torch.randn(512, 1536, device="cuda", generator=gen)).bfloat16()
    u0 = torch.randn(512, 1536, device="cuda", generator=gen).bfloat16()
    dh = torch.randn(512, 1536, device="cuda", generator=gen).bfloat16()
    res = []
    for fused in (False, True):
        g, u = g0.clone().requires_grad_(True), u0.clone().requires_grad_(True)
        h = SwiGLUFn.apply(g, u) if fused else torch.nn.functional.silu(g) * u
        h.backward(dh)
        res.append((h.detach(), g.grad.detach(), u.grad.detach()))
    assert _max_ulp(res[1][0], res[0][0]) <= 1
    assert _rel(res[1][1], res[0][1]) < 1e-2
    assert _max_ulp(res[1][2], res[0][2]) <= 1


def test_qat_step_with_fused_modules_tracks_eager():
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    dev = torch.device("cuda")
    curves = {}
    for fused in (False, True):
        step = qat.QatStep(spec, dev, backend="nvfp4", seed=0, fused=fused)
        curves[fused] = [float(step.step(qat.random_tokens(8, 256, spec.vocab, seed=10 + i, device=dev))[0])
                         for i in range(20)]
    for a, b in zip(curves[True], curves[False]):
        assert abs(a - b) / b < 5e-3, (a, b)


@pytest.mark.parametrize("rows,vocab", [(64, 49152), (37, 1000), (5, 8)])
def test_cross_entropy_kernel_matches_torch(rows, vocab):
    """cdlb200_cross_entropy against the torch chunk step it replaces: fp32
    log-sum-exp of the bf16 logits, per-row loss, bf16 (softmax - onehot) / n.
    Row 1 carries an ignored target (-100): zero loss and zero gradient."""
    import numpy as np

    from cdl_b200 import _lib

    gen = torch.Generator("cuda").manual_seed(rows + vocab)
    logits = (torch.randn(rows, vocab, device="cuda", generator=gen) * 3).bfloat16()
    targets = torch.randint(0, vocab, (rows,), device="cuda", generator=gen)
    if rows > 1:
        targets[1] = -100
    n = 4 * rows + 3
    ref = logits.float()
    lse = torch.logsumexp(ref, dim=1)
    valid = targets >= 0
    safe_t = targets.clamp_min(0)
    ref_loss = torch.where(valid, lse - ref.gather(1, safe_t[:, None])[:, 0], torch.zeros_like(lse))
    p = (ref - lse[:, None]).exp()
    p[torch.arange(rows, device="cuda")[valid], targets[valid]] -= 1.0
    p[~valid] = 0.0
    ref_grad = p.div_(n).bfloat16()

    out = logits.clone()
    loss = torch.empty(rows, dtype=torch.float32, device="cuda")
    _lib.call("cdlb200_cross_entropy", _lib.ptr(out), _lib.ptr(targets), rows, vocab,
              float(np.float32(1.0) / np.float32(n)), _lib.ptr(loss), _lib.stream(out.device))
    torch.cuda.synchronize()
    assert torch.allclose(loss, ref_loss, rtol=1e-5, atol=1e-5)
    assert _max_ulp(out, ref_grad) <= 1
    differ = float((out != ref_grad).float().mean())
    print("cross entropy: elements differing by one bf16 step", differ)
    assert differ < 1e-3
    if rows > 1:
        assert float(out[1].float().abs().max()) == 0.0 and float(loss[1]) == 0.0


def test_linear_cross_entropy_matches_plain_loss():
    """Chunked LinearCrossEntropy (kernel per chunk) against plain fp32-logit
    cross entropy with autograd: loss and both gradients."""
    from cdl_b200.train.qat import LinearCrossEntropy

    gen = torch.Generator("cuda").manual_seed(7)
    n, d, v = 3000, 256, 4096
    h = (torch.randn(n, d, device="cuda", generator=gen)).bfloat16().requires_grad_()
    w = (torch.randn(v, d, device="cuda", generator=gen) * 0.05).bfloat16().requires_grad_()
    t = torch.randint(0, v, (n,), device="cuda", generator=gen)
    loss = LinearCrossEntropy.apply(h, w, t, 1024)
    loss.backward()
    h2, w2 = h.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    ref = torch.nn.functional.cross_entropy((h2 @ w2.t()).float(), t)
    ref.backward()
    assert abs(float(loss.detach()) - float(ref.detach())) < 1e-4 * float(ref.detach())
    assert _rel(h.grad, h2.grad) < 1e-2
    assert _rel(w.grad, w2.grad) < 1e-2


@pytest.mark.parametrize("scale", [1.0, 0.5, 0.3, -2.0])
def test_scale_kernel_matches_torch_multiply(scale):
    """``cdlb200_scale_bf16`` (the in-place grad_output scaling of the fused
    linear cross entropy's backward) gives torch's bf16 product bit for bit;
    with a scale of 1 it leaves x as it is."""
    from cdl_b200 import _lib

    g = torch.Generator().manual_seed(4)
    x = (torch.randn(1000, 264, generator=g) * 3).bfloat16()
    x[0, :4] = torch.tensor([0.0, -0.0, float("inf"), 1e-40])
    x = x.cuda()
    s = torch.tensor([scale], dtype=torch.bfloat16, device="cuda")
    want = x * s
    got = x.clone()
    _lib.call("cdlb200_scale_bf16", _lib.ptr(got), got.numel(), _lib.ptr(s), _lib.stream(got.device))
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_linear_cross_entropy_backward_scales_by_grad_output():
    """The chunked loss's gradients under ``(loss * c).backward()`` are c times
    those of ``loss.backward()`` (c a power of two: exact in bf16)."""
    from cdl_b200.train import qat

    g = torch.Generator().manual_seed(5)
    h0 = (torch.randn(512, 256, generator=g) * 0.5).bfloat16().cuda()
    w0 = (torch.randn(1024, 256, generator=g) * 0.05).bfloat16().cuda()
    t = torch.randint(0, 1024, (512,), generator=g).cuda()
    grads = []
    for c in (1.0, 0.25):
        h, w = h0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        (qat.LinearCrossEntropy.apply(h, w, t, 256) * c).backward()
        grads.append((h.grad, w.grad))
    for a, b in zip(grads[0], grads[1]):
        assert torch.equal((a * 0.25).view(torch.int16), b.view(torch.int16))


def test_epilogue_amax_feeds_single_pass_encode():
    """RMSNorm and SwiGLU outputs carry their global amax; the NVFP4 encode of
    such an activation (one pass, with the dequantized copy) equals the
    two-pass quantizer and the dequantizer bit for bit."""
    from cdl_b200.core.kernel.dequant import nvfp4_dequant
    from cdl_b200.core.kernel.quant import nvfp4_quant
    from cdl_b200.model.components.fused import AMAX_ATTR, RMSNormFn, SwiGLUFn
    from cdl_b200.model.components.quant.ste import SteTensor

    gen = torch.Generator("cuda").manual_seed(11)
    x = torch.randn(256, 512, device="cuda", generator=gen).bfloat16()
    w = (1 + 0.1 * torch.randn(512, device="cuda", generator=gen)).bfloat16()
    g = torch.randn(384, 1024, device="cuda", generator=gen).bfloat16()
    u = torch.randn(384, 1024, device="cuda", generator=gen).bfloat16()
    for out in (RMSNormFn.apply(x, w, 1e-5), SwiGLUFn.apply(g, u)):
        owner = out._base if out._base is not None else out
        amax, _ = getattr(owner, AMAX_ATTR)
        want = int((out.contiguous().view(torch.int16).int() & 0x7FFF).max())
        assert int(amax.max().item()) == want
        st = SteTensor(theta=out.reshape(-1, out.shape[-1]), simulation=None)
        p, s, a = st.encode_swizzled("nvfp4")
        d = st.cached_dequant("nvfp4")
        assert d is not None
        rp, rs, ra = nvfp4_quant(out.reshape(-1, out.shape[-1]).contiguous(), swizzled=True)
        assert torch.equal(p, rp) and torch.equal(s, rs) and torch.equal(a.reshape(-1), ra.reshape(-1))
        assert torch.equal(d, nvfp4_dequant(rp, rs, ra, swizzled=True))


def test_swiglu_backward_gradient_amax():
    """The SwiGLU backward forms the amax words of dg and du; they are found
    again through the engine's reshape views of the gradients, and the dual
    encode given them equals the one that computes its own amax."""
    from cdl_b200.core.kernel.quant import nvfp4_dual_quant
    from cdl_b200.model.components.fused import SwiGLUFn, grad_amax

    gen = torch.Generator("cuda").manual_seed(12)
    g = torch.randn(2, 128, 1024, device="cuda", generator=gen).bfloat16().requires_grad_()
    u = torch.randn(2, 128, 1024, device="cuda", generator=gen).bfloat16().requires_grad_()
    dh = torch.randn(2, 128, 1024, device="cuda", generator=gen).bfloat16()
    seen = {}
    g.register_hook(lambda t: seen.__setitem__("g", t))
    u.register_hook(lambda t: seen.__setitem__("u", t))
    SwiGLUFn.apply(g, u).backward(dh)
    for name in ("g", "u"):
        grad = seen[name]
        words = grad_amax(grad.reshape(-1, 1024))
        assert words is not None
        want = int((grad.contiguous().view(torch.int16).int() & 0x7FFF).max())
        assert int(words.max().item()) == want
        row, col = nvfp4_dual_quant(grad.reshape(-1, 1024), amax=words)
        row2, col2 = nvfp4_dual_quant(grad.reshape(-1, 1024))
        for a, b in zip(row + col, row2 + col2):
            assert torch.equal(a, b)
    other = torch.zeros(256, 1024, device="cuda", dtype=torch.bfloat16)
    assert grad_amax(other) is None
    # rotary backward: the q / k projection's gradient, [B, S, H * D] as the
    # linear's backward sees it
    from cdl_b200.model.components.fused import RopeFn

    base = torch.randn(2, 128, 4, 64, device="cuda", generator=gen).bfloat16().requires_grad_()
    ang = torch.randn(1, 128, 32, device="cuda", generator=gen)
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16().contiguous()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16().contiguous()
    base.register_hook(lambda t: seen.__setitem__("q", t))
    RopeFn.apply(base.transpose(1, 2), cos, sin).backward(
        torch.randn(2, 4, 128, 64, device="cuda", generator=gen).bfloat16())
    gq = seen["q"].reshape(-1, 256)
    words = grad_amax(gq)
    assert words is not None
    assert int(words.max().item()) == int((gq.contiguous().view(torch.int16).int() & 0x7FFF).max())
    seen["g"].add_(1)  # written after the kernel: its words no longer hold
    assert grad_amax(seen["g"].reshape(-1, 1024)) is None


@pytest.mark.parametrize("rows,d", [(8192, 2048), (4096, 576), (333, 64)])
def test_rmsnorm_backward_is_deterministic(rows, d):
    """The weight gradient's fp32 partial sums are folded in a fixed order
    (row slots of a CTA one after another, then the CTAs' rows by one column
    kernel), so repeated backwards give the same bits.  d = 2048 and 576 run
    two and four row slots per CTA, d = 64 eight."""
    from cdl_b200.model.components.fused import RMSNormFn

    gen = torch.Generator("cuda").manual_seed(d + 1)
    w = (1.0 + 0.1 * torch.randn(d, device="cuda", generator=gen)).bfloat16()
    x = (3.0 * torch.randn(rows, d, device="cuda", generator=gen)).bfloat16()
    dy = torch.randn(rows, d, device="cuda", generator=gen).bfloat16()
    outs = []
    for _ in range(4):
        xx, ww = x.clone().requires_grad_(), w.clone().requires_grad_()
        RMSNormFn.apply(xx, ww, 1e-5).backward(dy)
        outs.append((xx.grad, ww.grad))
    for dx, dw in outs[1:]:
        assert torch.equal(dx, outs[0][0]) and torch.equal(dw, outs[0][1])


@pytest.mark.parametrize("rows,d", [(1000, 576), (300, 2048), (8, 64)])
def test_residual_rmsnorm_matches_add_then_rmsnorm(rows, d):
    """The fused residual add + RMSNorm equals a bf16 add followed by the
    RMSNorm kernel, forward bit for bit; its backward equals the norm's input
    gradient plus the residual gradient as autograd sums them, and carries
    that gradient's amax."""
    from cdl_b200.model.components.fused import ResidualRMSNormFn, RMSNormFn, grad_amax

    gen = torch.Generator("cuda").manual_seed(rows * 3 + d)
    w = (1.0 + 0.1 * torch.randn(d, device="cuda", generator=gen)).bfloat16()
    res = (2.0 * torch.randn(2, rows, d, device="cuda", generator=gen)).bfloat16()
    x = torch.randn(2, rows, d, device="cuda", generator=gen).bfloat16()
    dh = torch.randn(2, rows, d, device="cuda", generator=gen).bfloat16()
    dy = torch.randn(2, rows, d, device="cuda", generator=gen).bfloat16()
    outs = []
    for fused in (False, True):
        r, xx = res.clone().requires_grad_(), x.clone().requires_grad_()
        ww = w.clone().requires_grad_()
        if fused:
            h, y = ResidualRMSNormFn.apply(r, xx, ww, 1e-5)
        else:
            h = r + xx
            y = RMSNormFn.apply(h, ww, 1e-5)
        seen = {}
        xx.register_hook(lambda t: seen.__setitem__("x", t))
        torch.autograd.backward([h, y], [dh, dy])
        outs.append((h.detach(), y.detach(), r.grad, xx.grad, ww.grad, seen["x"]))
    (h0, y0, dr0, dx0, dw0, _), (h1, y1, dr1, dx1, dw1, sx) = outs
    assert torch.equal(h1, h0) and torch.equal(y1, y0)
    assert torch.equal(dr1, dr0) and torch.equal(dx1, dx0)
    assert torch.equal(dw1, dw0)  # same grid, partial sums folded in a fixed order
    words = grad_amax(sx.reshape(-1, d))
    assert words is not None
    assert int(words.max().item()) == int((dx1.view(torch.int16).int() & 0x7FFF).max())


def test_fused_decoder_loop_matches_layer_by_layer():
    """The patched LlamaModel loop (residual adds fused into the norms) gives
    the same loss as transformers' decoder loop over the same fused modules,
    and gradients within float noise."""
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    ids = qat.random_tokens(2, 64, spec.vocab, seed=3, device=torch.device("cuda"))
    res = []
    for fuse in (False, True):
        model = qat.build_model(spec, torch.device("cuda"), seed=1, fused=False)
        from cdl_b200.model.components.fused import patch_llama

        patch_llama(model, fuse_residual=fuse)
        hidden = model.model(input_ids=ids, use_cache=False).last_hidden_state
        loss = hidden.float().square().mean()
        loss.backward()
        res.append((hidden.detach(), {n: p.grad.detach().clone() for n, p in model.named_parameters()}))
    (h0, g0), (h1, g1) = res
    assert torch.equal(h1, h0)
    for n in g0:
        assert _rel(g1[n], g0[n]) < 2e-2, n
