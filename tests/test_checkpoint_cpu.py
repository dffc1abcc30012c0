"""Checkpoint dictionary format (cdl_b200.train.checkpoint) on CPU with
torch's AdamW: keys, atomic write, resume restores model, optimizer,
scheduler and RNG streams."""

import random

import torch

from cdl_b200.train.checkpoint import load_checkpoint, save_checkpoint


def _setup():
    torch.manual_seed(0)
    model = torch.nn.Linear(8, 4)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-2)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: min(1.0, (s + 1) / 3))
    return model, opt, sched


def _train(model, opt, sched, n):
    for _ in range(n):
        loss = model(torch.randn(2, 8)).square().sum()
        loss.backward()
        opt.step()
        sched.step()
        opt.zero_grad()


def test_checkpoint_round_trip(tmp_path):
    model, opt, sched = _setup()
    _train(model, opt, sched, 3)
    save_checkpoint(tmp_path / "last.ckpt", model, opt, sched, epoch=2, global_step=3)
    assert not (tmp_path / "last.ckpt.tmp").exists()
    ck = torch.load(tmp_path / "last.ckpt", weights_only=False)
    assert set(ck) == {"epoch", "global_step", "model", "optimizer", "lr_scheduler", "rng"}
    assert set(ck["rng"]) == {"python", "torch", "cuda"}
    py_next = random.random()
    _train(model, opt, sched, 2)
    want = [p.detach().clone() for p in model.parameters()]

    model2, opt2, sched2 = _setup()
    epoch, step = load_checkpoint(tmp_path, model2, opt2, sched2, torch.device("cpu"))
    assert (epoch, step) == (3, 3) and random.random() == py_next
    _train(model2, opt2, sched2, 2)
    for a, b in zip(want, model2.parameters()):
        assert torch.equal(a, b.detach())
