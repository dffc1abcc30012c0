"""The data-parallel QAT step captured in one CUDA graph per step, over NCCL on
two GPUs (one process each): the all-reduces issued from the backward hooks
are captured with the rest of the step, and replaying the graph leaves every
rank with the same parameters as the eager data-parallel step on the same
batches.  Needs two GPUs; skipped otherwise."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SPEC, BATCH, SEQ, STEPS = "tiny", 2, 128, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from cdl_b200.train import qat

    spec = qat.SPECS[SPEC]
    ids = qat.random_tokens(BATCH * world * STEPS, SEQ, spec.vocab, seed=7, device=dev)
    batches = [ids[(s * world + rank) * BATCH:(s * world + rank + 1) * BATCH] for s in range(STEPS)]
    out = {}
    for graph in (False, True):
        step = qat.QatStep(spec, dev, backend="nvfp4_qbwd", lr=1e-3, seed=0, ddp=True, graph=graph,
                           init_device="cpu")
        if not graph:  # the graph step's three warm-up steps on the first batch
            for _ in range(3):
                step.step(batches[0])
        losses, norms = [], []
        for b in batches:
            loss, gn = step.step(b)
            losses.append(float(loss))
            norms.append(float(gn))
        step.check_status()
        flat = torch.cat([p.detach().float().reshape(-1) for p in step.model.parameters()]).cpu()
        out["graph" if graph else "eager"] = {"params": flat, "losses": losses, "norms": norms}
        step.release_graph()
        step.sync.remove()
        del step
    torch.save(out, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_graph_captured_data_parallel_step_matches_eager(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for mode in ("eager", "graph"):
        # the all-reduce hands every rank the same gradient sums
        assert torch.equal(res[0][mode]["params"], res[1][mode]["params"]), mode
        assert res[0][mode]["norms"] == res[1][mode]["norms"], mode
    e, g = res[0]["eager"], res[0]["graph"]
    print(f"eager losses {e['losses']} graph {g['losses']}; norms {e['norms']} / {g['norms']}")
    # the graph (three warm-up steps and the capture on the first batch, then
    # replays) follows the eager step on the same sequence of batches
    for a, b in zip(e["losses"], g["losses"]):
        assert abs(a - b) <= 5e-3 * abs(a), (a, b)
    for a, b in zip(e["norms"], g["norms"]):
        assert abs(a - b) <= 5e-2 * abs(a), (a, b)
    diff = (e["params"] - g["params"]).abs()
    assert float(diff.mean()) < 1e-3, float(diff.mean())
