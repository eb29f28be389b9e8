"""Shared helpers for the tests: seeded inputs and the error metrics."""
from __future__ import annotations

import numpy as np
import torch

# Parity bar for the 16-bit GEMM outputs against the oracle:
#   max relative error  max_i |y_i - r_i| / max(|r_i|, 0.01 * rms(r))  <= 1e-2
#   mean absolute error mean_i |y_i - r_i|                              <= 1e-3
# The floor keeps outputs that cancel to ~0 from dominating; one 16-bit ulp
# of a normal value is <= 2**-7 relative (bf16), below the 1e-2 bar.
MAX_REL = 1e-2
MAE = 1e-3

TORCH_DT = {0: torch.float16, 1: torch.bfloat16}
DT_CODE = {torch.float16: 0, torch.bfloat16: 1}


from orininfer_b200.synth import seeded  # noqa: F401  (x ~ N(0, scale^2), seeded, 16-bit)


def bits(t: torch.Tensor) -> np.ndarray:
    """uint16 bit patterns of a 16-bit CPU tensor."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype)


def errors(y, r) -> tuple[float, float]:
    y = torch.as_tensor(y).double().flatten()
    r = torch.as_tensor(r).double().flatten()
    d = (y - r).abs()
    rms = r.pow(2).mean().sqrt().item() if r.numel() else 0.0
    floor = max(0.01 * rms, 1e-30)
    max_rel = (d / r.abs().clamp_min(floor)).max().item() if r.numel() else 0.0
    return max_rel, d.mean().item() if r.numel() else 0.0


def assert_close(y, r, what: str = "", max_rel: float = MAX_REL, mae: float = MAE) -> None:
    y = torch.as_tensor(y)
    r = torch.as_tensor(r)
    assert torch.isfinite(y.double()).all(), f"{what}: non-finite output"
    mr, ma = errors(y, r)
    assert mr <= max_rel and ma <= mae, f"{what}: max_rel={mr:.3e} (<= {max_rel}), mae={ma:.3e} (<= {mae})"
