"""Seeded synthetic tensors (the benchmarks use random-init weights: no
checkpoint is read).  Draw order and scale follow the workload definitions:
fp32 N(0, scale^2) from torch.manual_seed(seed) on the CPU, then cast."""
from __future__ import annotations

import torch


def seeded(shape, seed: int, scale: float = 1.0, dtype=torch.float16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * scale).to(dtype)
