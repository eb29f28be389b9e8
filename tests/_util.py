"""Shared helpers for the tests: seeded inputs and the error metrics."""
from __future__ import annotations

import numpy as np
import torch

# Parity bar for the GEMM outputs against the oracle (same 16-bit inputs):
#   max relative error  max_i |y_i - r_i| / max_i |r_i|   <= 1e-2
#   mean absolute error mean_i |y_i - r_i|                <= 1e-3
#   and, for 16-bit outputs of one GEMM, at least 95% of them bit-identical
#   (both sides accumulate in fp32; only the summation order differs, which
#   flips a final rounding for well under 1% of outputs).
# The relative error is taken against the largest output: the reference
# rounds the accumulator before the residual add (round16(x + round16(acc))),
# so where x and acc cancel a one-ulp flip of round16(acc) is an absolute
# error of ulp(acc) on an output near zero, and an elementwise ratio there
# says nothing about the kernel.
MAX_REL = 1e-2
MAE = 1e-3
EXACT_MIN = 0.95
# Beside the normwise figure, the elementwise relative error
#   max_i |y_i - r_i| / |r_i|  over the outputs with |r_i| >= ELEM_FLOOR * max_j |r_j|
# is computed for every comparison and reported in the assertion messages.  A
# one-unit flip of a 16-bit rounding is at most 2^-8 (fp16 2^-11) of the value,
# so for a plain GEMM it stays under 1e-2; callers that check it pass elem_max.
# It is not asserted by default: with the residual epilogue the reference's
# rounding of acc before the add puts ulp(acc) on outputs that cancel to far
# below |acc|, which no floor short of |acc| itself excludes.
ELEM_FLOOR = 1e-2
# The 1e-2 elementwise bar is fp16's (the path's own dtype).  bf16 keeps 8
# significand bits to fp16's 11, so one unit is up to 2^-7 of a value: where
# both sides' roundings of g and u (SwiGLU) and of the output flip by one
# unit, outputs differ by up to three of them.  bf16 comparisons are held to
# that, three units.
ELEM_MAX_BF16 = 3 * 2.0 ** -7


def elem_max_for(dt: int) -> float:
    """Elementwise relative-error bound for 16-bit outputs of dtype code dt."""
    return MAX_REL if dt == 0 else ELEM_MAX_BF16

TORCH_DT = {0: torch.float16, 1: torch.bfloat16}
DT_CODE = {torch.float16: 0, torch.bfloat16: 1}


from orininfer_b200.synth import seeded  # noqa: F401  (x ~ N(0, scale^2), seeded, 16-bit)


def bits(t: torch.Tensor) -> np.ndarray:
    """uint16 bit patterns of a 16-bit CPU tensor."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype)


def errors(y, r) -> tuple[float, float, float]:
    """(normwise max relative error, mean absolute error, fraction exactly equal)."""
    y = torch.as_tensor(y).double().flatten()
    r = torch.as_tensor(r).double().flatten()
    if r.numel() == 0:
        return 0.0, 0.0, 1.0
    d = (y - r).abs()
    scale = max(r.abs().max().item(), 1e-30)
    return d.max().item() / scale, d.mean().item(), (d == 0).double().mean().item()


def elementwise_rel(y, r, floor: float = ELEM_FLOOR) -> float:
    """max_i |y_i - r_i| / |r_i| over the outputs with |r_i| >= floor * max|r|."""
    y = torch.as_tensor(y).double().flatten()
    r = torch.as_tensor(r).double().flatten()
    if r.numel() == 0:
        return 0.0
    a = r.abs()
    keep = a >= floor * max(a.max().item(), 1e-30)
    if not bool(keep.any()):
        return 0.0
    return ((y - r).abs()[keep] / a[keep]).max().item()


def assert_close(y, r, what: str = "", max_rel: float = MAX_REL, mae: float = MAE,
                 exact_min: float | None = None,
                 elem_max: float | None = None) -> tuple[float, float, float]:
    """Normwise relative error, mean absolute error and (optionally) the share of
    bit-identical outputs and the elementwise relative error against their
    bounds; the elementwise figure is always part of the message."""
    y = torch.as_tensor(y)
    r = torch.as_tensor(r)
    assert torch.isfinite(y.double()).all(), f"{what}: non-finite output"
    mr, ma, ex = errors(y, r)
    er = elementwise_rel(y, r)
    msg = (f"{what}: max_rel={mr:.3e} (<= {max_rel}), mae={ma:.3e} (<= {mae}), exact={ex:.4f}, "
           f"elementwise_rel={er:.3e} (|r| >= {ELEM_FLOOR} max|r|)")
    assert mr <= max_rel and ma <= mae, msg
    if exact_min is not None:
        assert ex >= exact_min, f"only {ex:.4f} of outputs bit-identical (>= {exact_min}); " + msg
    if elem_max is not None:
        assert er <= elem_max, f"elementwise_rel above {elem_max}; " + msg
    return mr, ma, ex
