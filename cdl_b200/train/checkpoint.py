"""Training checkpoints in the dictionary format of cdl's ``checkpoint.py``
(cdl/checkpoint.py:12-64), so that a run can resume from a checkpoint either
side wrote:

    {"epoch", "global_step", "model" (state_dict of the unwrapped model),
     "optimizer" (torch.optim.AdamW's state_dict layout), "lr_scheduler",
     "rng": {"python", "torch", "cuda"}}

written to ``<path>.tmp`` and renamed over ``path``.  ``ClipAdamW``
(cdl_b200.train.optim) reads and writes the AdamW layout.
"""

from __future__ import annotations

import logging
import os
import random
from pathlib import Path

import torch
from torch import nn

logger = logging.getLogger(__name__)


def into_orig_mod(model: nn.Module) -> nn.Module:
    """The module under a ``torch.compile`` wrapper (``_orig_mod``) or DDP (``module``)."""
    model = getattr(model, "_orig_mod", model)
    return model.module if isinstance(model, nn.parallel.DistributedDataParallel) else model


def save_checkpoint(path: Path, model: nn.Module, optimizer, lr_scheduler, epoch: int, global_step: int) -> None:
    """``lr_scheduler`` may be None (no schedule): its entry is then empty."""
    path = Path(path)
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save({
        "epoch": epoch,
        "global_step": global_step,
        "model": into_orig_mod(model).state_dict(),
        "optimizer": optimizer.state_dict(),
        "lr_scheduler": lr_scheduler.state_dict() if lr_scheduler is not None else {},
        "rng": {
            "python": random.getstate(),
            "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None,
        },
    }, tmp)
    os.replace(tmp, path)
    logger.info("checkpoint saved to %s", path)


def load_checkpoint(resume_dir: Path, model: nn.Module, optimizer, lr_scheduler,
                    device: torch.device) -> tuple[int, int]:
    """Restore ``resume_dir/last.ckpt``; returns (next epoch, global step).
    ``lr_scheduler`` may be None (no schedule)."""
    ckpt = torch.load(Path(resume_dir) / "last.ckpt", map_location=device, weights_only=False)
    into_orig_mod(model).load_state_dict(ckpt["model"])
    optimizer.load_state_dict(ckpt["optimizer"])
    if lr_scheduler is not None:
        lr_scheduler.load_state_dict(ckpt["lr_scheduler"])
    random.setstate(ckpt["rng"]["python"])
    torch.set_rng_state(ckpt["rng"]["torch"].cpu())
    if torch.device(device).type == "cuda" and ckpt["rng"]["cuda"] is not None:
        torch.cuda.set_rng_state_all([s.cpu() for s in ckpt["rng"]["cuda"]])
    logger.info("checkpoint loaded from %s", resume_dir)
    return ckpt["epoch"] + 1, ckpt["global_step"]
