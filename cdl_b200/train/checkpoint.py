"""Training checkpoints in cdl's dictionary format (cdl/checkpoint.py:12-64),
so that a run resumes from a file either side wrote.

The format is a flat ``torch.save`` dictionary:

=================  ==========================================================
``epoch``          int, the epoch the checkpoint was taken in
``global_step``    int, optimizer steps taken
``model``          ``state_dict`` of the bare model (no compile / DDP wrapper)
``optimizer``      ``state_dict`` in ``torch.optim.AdamW``'s layout
                   (``ClipAdamW`` in ``cdl_b200.train.optim`` reads and
                   writes it too)
``lr_scheduler``   the scheduler's ``state_dict``; ``{}`` without a schedule
``rng``            ``{"python", "torch", "cuda"}``: the three generator
                   states (``cuda`` is None on a host without CUDA)
=================  ==========================================================

A file is written next to its destination (``<name>.tmp``) and renamed over
it, so a crash never leaves a half-written checkpoint under the real name.
Resuming reads ``<dir>/last.ckpt`` and continues with the next epoch.
"""

from __future__ import annotations

import logging
import os
import random
from pathlib import Path

import torch
from torch import nn

logger = logging.getLogger(__name__)

KEYS = ("epoch", "global_step", "model", "optimizer", "lr_scheduler", "rng")
LAST = "last.ckpt"


def into_orig_mod(model: nn.Module) -> nn.Module:
    """The module whose ``state_dict`` is stored: unwraps ``torch.compile``
    (``_orig_mod``) and ``DistributedDataParallel`` (``module``), in any order."""
    while True:
        if hasattr(model, "_orig_mod"):
            model = model._orig_mod
        elif isinstance(model, nn.parallel.DistributedDataParallel):
            model = model.module
        else:
            return model


def _rng_snapshot() -> dict:
    cuda = torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None
    return {"python": random.getstate(), "torch": torch.get_rng_state(), "cuda": cuda}


def _rng_restore(rng: dict, device: torch.device) -> None:
    random.setstate(rng["python"])
    torch.set_rng_state(rng["torch"].cpu())
    if torch.device(device).type == "cuda" and rng.get("cuda") is not None:
        torch.cuda.set_rng_state_all([s.cpu() for s in rng["cuda"]])


def save_checkpoint(path: Path, model: nn.Module, optimizer, lr_scheduler, epoch: int, global_step: int) -> None:
    """Write the checkpoint of this point of training to ``path`` (atomically).
    ``lr_scheduler`` may be None (constant learning rate)."""
    path = Path(path)
    state = dict(zip(KEYS, (
        epoch,
        global_step,
        into_orig_mod(model).state_dict(),
        optimizer.state_dict(),
        {} if lr_scheduler is None else lr_scheduler.state_dict(),
        _rng_snapshot(),
    )))
    partial = path.parent / (path.name + ".tmp")
    torch.save(state, partial)
    os.replace(partial, path)
    logger.info("checkpoint saved to %s", path)


def load_checkpoint(resume_dir: Path, model: nn.Module, optimizer, lr_scheduler,
                    device: torch.device) -> tuple[int, int]:
    """Restore model, optimizer, scheduler (if any) and the generators from
    ``resume_dir/last.ckpt``; returns ``(epoch to start, global step)``."""
    state = torch.load(Path(resume_dir) / LAST, map_location=device, weights_only=False)
    missing = [k for k in KEYS if k not in state]
    if missing:
        raise KeyError(f"{Path(resume_dir) / LAST} is not a training checkpoint (missing {missing})")
    into_orig_mod(model).load_state_dict(state["model"])
    optimizer.load_state_dict(state["optimizer"])
    if lr_scheduler is not None:
        lr_scheduler.load_state_dict(state["lr_scheduler"])
    _rng_restore(state["rng"], device)
    logger.info("checkpoint loaded from %s", resume_dir)
    return state["epoch"] + 1, state["global_step"]
