"""Seeded synthetic inputs for the benchmark configurations.

The reference measures on synthetic data only (random tensors, random-init
models, uniform random tokens); these generators reproduce those shapes and
value distributions:

* ``c1_nvfp4``: one 4096x4096 bf16 tensor, N(0,1) from seed 0, with 0.1% of the
  entries (uniformly chosen) scaled x20 as outliers.
* ``c2_mx``: bf16 activations ``[rows, k]``, N(0,1) with a per-row standard
  deviation drawn log-uniform in [0.1, 10].
* ``c3_gemm``: A = bf16 N(0,1) activations ``[M, K]``, B = weights N(0, 0.02)
  ``[N, K]``.

Every generator runs on the CPU generator by default so the same seed gives
the same tensor on every machine; pass ``device="cuda"`` for large benchmark
inputs where only the distribution matters.
"""

from __future__ import annotations

import math

import torch


def _gen(seed: int, device: str) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def c1_nvfp4(rows: int = 4096, k: int = 4096, seed: int = 0, device: str = "cpu") -> torch.Tensor:
    g = _gen(seed, device)
    x = torch.randn(rows, k, generator=g, device=device, dtype=torch.float32)
    n = x.numel()
    idx = torch.randperm(n, generator=g, device=device)[: n // 1000]
    x.view(-1)[idx] *= 20.0
    return x.to(torch.bfloat16)


def c2_mx(rows: int = 16384, k: int = 2048, seed: int = 0, device: str = "cpu") -> torch.Tensor:
    g = _gen(seed, device)
    u = torch.rand(rows, 1, generator=g, device=device, dtype=torch.float32)
    std = torch.exp(math.log(0.1) + u * (math.log(10.0) - math.log(0.1)))
    x = torch.randn(rows, k, generator=g, device=device, dtype=torch.float32) * std
    return x.to(torch.bfloat16)


def c3_gemm(m: int, n: int, k: int, seed: int = 0, device: str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    g = _gen(seed, device)
    a = torch.randn(m, k, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    return a, w


def token_batches(batch: int, seq: int, vocab: int, seed: int, steps: int):
    """``steps`` batches of uniform random token ids ``[batch, seq]`` (int64,
    CPU), drawn one after another from one CPU generator seeded with ``seed``:
    the same sequence of batches on every machine."""
    g = _gen(seed, "cpu")
    for _ in range(steps):
        yield torch.randint(0, vocab, (batch, seq), generator=g, dtype=torch.int64)


C3_SHAPES = [(8192, 8192, 8192)] + [
    (m, n, k) for m in (2048, 16384) for (n, k) in ((2048, 8192), (8192, 2048), (49152, 576))
]
