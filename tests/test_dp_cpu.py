"""Data-parallel step logic on CPU ranks (gloo): DDP-averaged gradients give
every rank the same parameters, equal to one process stepping on the whole
batch, also with gradient accumulation over micro-batches; a failing rank surfaces as an error, not a hang."""

import os
import socket

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


def _worker(rank, world, port, out_dir, fail_rank, accum=False):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    step = qat.QatStep(spec, torch.device("cpu"), backend="none", lr=1e-3, seed=0, ddp=True)
    ids = qat.random_tokens(4, 32, spec.vocab, seed=7, device=torch.device("cpu"))
    mine = ids[rank * 2:(rank + 1) * 2]
    if rank == fail_rank:
        raise RuntimeError("injected rank failure")
    for _ in range(2):
        # accum: two micro-batches of one sequence each
        step.step([mine[:1], mine[1:]] if accum else mine)
    flat = torch.cat([p.detach().float().reshape(-1) for p in step.model.parameters()])
    torch.save(flat, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("accum", [False, True])
def test_ddp_two_ranks_match_single_process(tmp_path, accum):
    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path), -1, accum), nprocs=2, join=True)
    p0 = torch.load(tmp_path / "rank0.pt")
    p1 = torch.load(tmp_path / "rank1.pt")
    assert torch.equal(p0, p1)
    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    single = qat.QatStep(spec, torch.device("cpu"), backend="none", lr=1e-3, seed=0)
    ids = qat.random_tokens(4, 32, spec.vocab, seed=7, device=torch.device("cpu"))
    for _ in range(2):
        single.step(ids)
    ps = torch.cat([p.detach().float().reshape(-1) for p in single.model.parameters()])
    # mean over ranks of per-rank mean losses == mean over the full batch (equal halves)
    assert torch.allclose(p0, ps, rtol=0, atol=2e-2)
    assert (p0 - ps).abs().mean() < 2e-4


def test_failed_rank_raises_instead_of_hanging(tmp_path):
    port = _free_port()
    with pytest.raises(Exception):
        mp.spawn(_worker, args=(2, port, str(tmp_path), 1), nprocs=2, join=True)
