"""Host-side checks of the CCDL / ECDL quantizer modules (no kernel calls):
construction, scale initialization from a weight, learning-rate groups."""

import math

import pytest
import torch

from cdl_b200.model.components.quant import ccdl as Q


def test_ccdl_weight_init_and_lr_groups():
    torch.manual_seed(0)
    w = (torch.randn(64, 96) * 0.02).bfloat16()
    m = Q.Nvfp4CascadedCdlQuantForWeight(w, torch.bfloat16, 2.0)
    assert m.initialized and m.theta_topk == 16 and m.q_topk == 126 and m.log_q.shape == (64, 6, 1)
    # q = bf16(block amax / 6), logarithm in bf16 (the weight's dtype)
    want = (w.reshape(64, 6, 16).abs().amax(-1, keepdim=True) / torch.tensor(6.0, dtype=torch.bfloat16))
    assert torch.equal(m.log_q.detach(), want.clamp_min(torch.finfo(torch.float32).tiny).log().float())
    assert torch.equal(m.log_q_init, m.log_q.detach())
    eta = 1e-3
    assert m.get_q_lr(eta) == pytest.approx(eta / math.sqrt(16 * 2 ** 3))
    assert m.get_alpha_lr(eta) == pytest.approx(eta / math.sqrt(64 * 96 * 2 ** 3))
    assert m.get_theta_kappa_lr(eta) == pytest.approx(eta / math.sqrt(64 * 96))
    assert m.get_q_kappa_lr(eta) == pytest.approx(eta / math.sqrt(64 * 6))
    a = Q.Mxfp8CascadedCdlQuantForActivation((1, 96), 5, 5, torch.bfloat16, 2.0)
    assert not a.initialized and a.log_q.shape == (1, 3, 1)
    assert a.get_q_lr(eta) == pytest.approx(eta / math.sqrt(32 * 2 ** 8))
    with pytest.raises(ValueError):
        Q.Nvfp4CascadedCdlQuantForActivation((1, 96), 17, 5, torch.bfloat16, 2.0)
    with pytest.raises(ValueError):
        Q.Nvfp4CascadedCdlQuantForActivation((1, 96), 5, 127, torch.bfloat16, 2.0)

    class M(Q.CascadedCdlQuantMixin):
        def __init__(self):
            super().__init__()
            self.w, self.a = m, a

    groups, params = M().cascaded_cdl_get_param_groups(eta, train_alpha=False, train_kappa=True)
    assert len(params) == 8 and not m.log_alpha.requires_grad
    lrs = sorted(g["lr"] for g in groups)
    assert all(g["weight_decay"] == 0.0 for g in groups) and len(lrs) == 6


def test_ecdl_mixin_groups():
    from torch import nn

    from cdl_b200.model.components.quant import ecdl as X

    class M(X.ExtendedCdlQuantMixin):
        def __init__(self):
            super().__init__()
            self.a = X.Nvfp4ExtendedCdlQuantForActivation((1, 64), 5, torch.bfloat16, 2.0)
            self.w = X.Mxfp8ExtendedCdlQuantForWeight(torch.zeros(32, 64), torch.bfloat16, 3.0)
            self.other = nn.Linear(4, 4)

    m = M()
    assert m.extended_cdl_get_activation_quant_counts() == 64
    assert m.extended_cdl_get_weight_quant_counts() == 32 * 64
    stats = m.extended_cdl_quant_stats()
    assert stats["a.kappa"] == pytest.approx(2.0) and stats["w.kappa"] == pytest.approx(3.0)
    groups, params = m.extended_cdl_get_param_groups(1e-3, train_kappa=True)
    assert len(groups) == 1 and len(groups[0]["params"]) == 2 and len(params) == 2
    groups, _ = m.extended_cdl_get_param_groups(1e-3, train_kappa=False)
    assert groups == [] and not m.a.log_kappa.requires_grad
