"""Data-parallel step logic on CPU ranks (gloo): gradients averaged by
``GradSync`` (the loss pre-scaled by 1 / world, summed over ranks) give
every rank the same parameters, equal to one process stepping on the whole
batch (world sizes 2, 4 and 8, also with gradient accumulation over
micro-batches); a late rank only delays the others; a NaN gradient on one
rank reaches every rank's gradient norm; a failing rank surfaces as an
error, not a hang."""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir, mode):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    step = qat.QatStep(spec, torch.device("cpu"), backend="none", lr=1e-3, seed=0, ddp=True)
    ids = qat.random_tokens(2 * world, 32, spec.vocab, seed=7, device=torch.device("cpu"))
    mine = ids[rank * 2:(rank + 1) * 2]
    if mode == "fail" and rank == 1:
        raise RuntimeError("injected rank failure")
    if mode == "delay" and rank == world - 1:
        time.sleep(3.0)  # arrives late at every collective of the first step
    if mode == "nan" and rank == 1:
        p = next(q for q in step.model.parameters() if q.requires_grad and q.ndim == 2)
        p.register_hook(lambda g: torch.full_like(g, float("nan")))
    norms = []
    for _ in range(2):
        # accum: two micro-batches of one sequence each
        _, gn = step.step([mine[:1], mine[1:]] if mode == "accum" else mine)
        norms.append(float(gn))
    flat = torch.cat([p.detach().float().reshape(-1) for p in step.model.parameters()])
    torch.save({"params": flat, "norms": norms}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _single(world):
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    single = qat.QatStep(spec, torch.device("cpu"), backend="none", lr=1e-3, seed=0)
    ids = qat.random_tokens(2 * world, 32, spec.vocab, seed=7, device=torch.device("cpu"))
    for _ in range(2):
        single.step(ids)
    return torch.cat([p.detach().float().reshape(-1) for p in single.model.parameters()])


@pytest.mark.parametrize("world,mode", [(2, "plain"), (2, "accum"), (4, "plain"), (8, "plain"), (4, "delay")])
def test_ddp_ranks_match_single_process(tmp_path, world, mode):
    port = _free_port()
    mp.spawn(_worker, args=(world, port, str(tmp_path), mode), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r in range(1, world):
        assert torch.equal(res[0]["params"], res[r]["params"])
        assert res[0]["norms"] == res[r]["norms"]
    ps = _single(world)
    # mean over ranks of per-rank mean losses == mean over the full batch (equal shares)
    assert torch.allclose(res[0]["params"], ps, rtol=0, atol=2e-2)
    assert (res[0]["params"] - ps).abs().mean() < 2e-4


def test_nan_gradient_on_one_rank_reaches_every_rank(tmp_path):
    """The all-reduce spreads a non-finite gradient to every rank, so every
    rank sees the same non-finite norm and can take the same decision."""
    import math

    world = 4
    port = _free_port()
    mp.spawn(_worker, args=(world, port, str(tmp_path), "nan"), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r in range(world):
        assert not math.isfinite(res[r]["norms"][0])


def test_failed_rank_raises_instead_of_hanging(tmp_path):
    port = _free_port()
    with pytest.raises(Exception):
        mp.spawn(_worker, args=(2, port, str(tmp_path), "fail"), nprocs=2, join=True)
