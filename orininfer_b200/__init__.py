"""orininfer_b200 — the B200 (sm_100a) linear-layer hot path of OrinInfer.

Importing the package loads liborin_b200.so (built in-tree by
``python -m orininfer_b200.build``) and fails if it is missing.
"""
from .kernels import (OrinError, add, bf16_to_fp32, device_check, fused_silu_mul, linear,
                      linear_into, matmul, pack_gate_up)

__all__ = [
    "OrinError", "add", "bf16_to_fp32", "device_check", "fused_silu_mul", "linear",
    "linear_into", "matmul", "pack_gate_up",
]
__version__ = "0.1.0"
