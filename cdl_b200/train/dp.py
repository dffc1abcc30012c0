"""Data-parallel gradient averaging for the QAT step, capturable in its CUDA graph.

cdl's training script runs on one GPU; the data-parallel step here (one
process per GPU, each on its own batch) averages the bf16 gradients over
ranks with NCCL all-reduces during the backward pass, the contract of
torch's ``DistributedDataParallel``: after ``loss.backward()`` every rank
holds the mean over ranks of its gradients.  ``GradSync`` keeps that contract
with less machinery, so that the whole data-parallel step (forward, backward,
the NCCL all-reduces, clipping and AdamW) is one CUDA graph per step, as the
single-GPU step is:

* a post-accumulate-grad hook on every trainable parameter issues that
  gradient's all-reduce (``async_op``) as soon as autograd has accumulated it
  for the last time in this backward pass, so the transfer runs on the process
  group's stream while the backward kernels of earlier layers are still
  running; the gradient is reduced in place (no bucket copy);
* ``finish()`` makes the current stream wait for every all-reduce issued,
  which is the join a graph capture needs before the optimizer reads the
  gradients;
* the number of accumulations per parameter and backward pass (two for the
  tied embedding: the LM head and the token lookup) is learnt from the first
  backward pass, whose all-reduces are issued at ``finish()`` in parameter
  order (a static graph, as ``DistributedDataParallel(static_graph=True)``
  assumes); every rank runs the same autograd graph, so the hooks fire, and
  the collectives are issued, in the same order on every rank;
* the mean is formed by scaling the loss by ``1 / world`` before the backward
  pass and summing: for a power-of-two world size the scaling is exact and
  every gradient equals, bit for bit, what DDP's divide-then-sum gives (the
  NVFP4 quantization of the gradients is invariant under a power-of-two
  scale: the global amax, the block scales and the codes scale together);
* with gradient accumulation only the last micro-batch's backward reduces
  (the earlier ones only accumulate locally), as DDP's ``no_sync`` does.

Parameters are broadcast from rank 0 at construction, as DDP does.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn


class GradSync:
    """All-reduces (sums) the gradients of ``params`` across the default process
    group from backward hooks.  Use as::

        sync.begin(reduce=True)
        (loss * sync.loss_scale).backward()
        sync.finish()
    """

    def __init__(self, params: list[nn.Parameter], group=None, broadcast: bool = True):
        if not dist.is_initialized():
            raise RuntimeError("GradSync needs an initialised torch.distributed process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.params = list(params)
        self.loss_scale = 1.0 / self.world
        self._index = {id(p): i for i, p in enumerate(self.params)}
        self._expected: list[int] | None = None
        self._counts = [0] * len(self.params)
        self._issued = [False] * len(self.params)
        self._works: list = []
        self._reduce = False
        self._active = False
        if broadcast:
            with torch.no_grad():
                for p in self.params:
                    dist.broadcast(p.data, 0, group=group)
        self._handles = [p.register_post_accumulate_grad_hook(self._hook) for p in self.params]

    def begin(self, reduce: bool = True) -> None:
        """Start a backward pass; ``reduce=False`` only accumulates locally."""
        if self._active:
            raise RuntimeError("GradSync.begin() twice without finish()")
        self._active = True
        self._reduce = reduce
        self._counts = [0] * len(self.params)
        self._issued = [False] * len(self.params)

    def _issue(self, i: int) -> None:
        g = self.params[i].grad
        if g is None:
            raise RuntimeError(f"parameter {i} has no gradient to reduce")
        self._works.append(dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
        self._issued[i] = True

    def _hook(self, p: nn.Parameter) -> None:
        if not self._active:
            return  # a backward pass outside begin() / finish(): no data-parallel semantics
        i = self._index[id(p)]
        self._counts[i] += 1
        if self._reduce and self._expected is not None:
            if self._counts[i] > self._expected[i]:
                raise RuntimeError("a gradient was accumulated after its all-reduce: the autograd graph "
                                   "changed between steps")
            if self._counts[i] == self._expected[i]:
                self._issue(i)

    def finish(self) -> None:
        """End the backward pass: issue the reductions not yet issued (all of
        them on the first pass), then make the current stream wait for every
        all-reduce.  After it each reduced ``.grad`` holds the sum over ranks."""
        if not self._active:
            raise RuntimeError("GradSync.finish() without begin()")
        try:
            if self._expected is None:
                self._expected = list(self._counts)
            if self._reduce:
                for i, c in enumerate(self._counts):
                    if c > 0 and not self._issued[i]:
                        self._issue(i)
            for w in self._works:
                w.wait()
        finally:
            self._works = []
            self._active = False

    def remove(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles = []
