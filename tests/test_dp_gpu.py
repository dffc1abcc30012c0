"""The data-parallel QAT step with the fused CUDA path, two ranks sharing one
GPU over gloo: the data-parallel gradient sync (``train/dp.py``) around the
fused decoder loop (residual adds in the norms), the quantized backward and
the fused optimizer leaves the same parameters on both ranks, close to one
process stepping on the whole batch.  (NCCL needs one GPU per rank; gloo
reduces the CUDA gradients through the host, which checks the same hooks.  No
kernel waits on another rank.)"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SPEC, BATCH, SEQ, STEPS = "tiny", 2, 128, 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir, backend):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from cdl_b200.train import qat

    spec = qat.SPECS[SPEC]
    dev = torch.device("cuda", 0)
    step = qat.QatStep(spec, dev, backend=backend, lr=1e-3, seed=0, ddp=True, init_device="cpu")
    ids = qat.random_tokens(BATCH * world, SEQ, spec.vocab, seed=7, device=dev)
    mine = ids[rank * BATCH:(rank + 1) * BATCH]
    norms = [float(step.step(mine)[1]) for _ in range(STEPS)]
    step.check_status()
    flat = torch.cat([p.detach().float().reshape(-1) for p in step.model.parameters()]).cpu()
    torch.save({"params": flat, "norms": norms}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("backend", ["nvfp4_qbwd", "nvfp4"])
def test_ddp_fused_step_on_one_gpu(tmp_path, backend):
    from cdl_b200.train import qat

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), backend), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert torch.equal(res[0]["params"], res[1]["params"])
    assert res[0]["norms"] == res[1]["norms"]
    # one process accumulating the gradients of the same two micro-batches:
    # each micro-batch is quantized with its own amax, as each rank's batch
    # is, and the gradient sync (the loss pre-scaled by 1 / world, a power of
    # two) sums the same two halves the accumulation adds, so the two runs
    # agree bit for bit (measured on B200, both backends).  Only the order of
    # a library's atomic reductions (attention backward) could move a weight;
    # the bound allows a few.  (Against one process on the whole batch the
    # amax differ, and AdamW's first steps, near sign(g), move every weight
    # whose quantized gradient changes sign by 2 lr per step.)
    spec = qat.SPECS[SPEC]
    dev = torch.device("cuda", 0)
    single = qat.QatStep(spec, dev, backend=backend, lr=1e-3, seed=0, init_device="cpu")
    ids = qat.random_tokens(BATCH * world, SEQ, spec.vocab, seed=7, device=dev)
    micro = [ids[r * BATCH:(r + 1) * BATCH] for r in range(world)]
    norms = [float(single.step(micro)[1]) for _ in range(STEPS)]
    ps = torch.cat([p.detach().float().reshape(-1) for p in single.model.parameters()]).cpu()
    diff = (res[0]["params"] - ps).abs()
    print(f"{backend}: norms ranks {res[0]['norms']} one process {norms}; "
          f"params mean diff {float(diff.mean()):.3e} max {float(diff.max()):.3e} "
          f"changed {float((diff > 0).float().mean()):.3e}")
    for a, b in zip(res[0]["norms"], norms):
        assert abs(a - b) <= 1e-2 * b, (a, b)
    assert float((diff > 0).float().mean()) < 1e-3
