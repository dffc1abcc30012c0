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
