"""orininfer_b200 — the B200 (sm_100a) linear-layer hot path of OrinInfer.

The first use of any operator loads liborin_b200.so (built in-tree by
``python -m orininfer_b200.build``) and raises ImportError if it is missing:
there is no CPU path.  ``orininfer_b200.build`` itself does not load it.
"""
import importlib

__all__ = [
    "OrinError", "add", "bf16_to_fp32", "device_check", "fused_silu_mul", "linear",
    "linear_into", "lm_head_argmax", "matmul", "pack_gate_up", "plan_info", "linear_workspace",
    "linear_workspace_bytes",
]
__version__ = "0.1.0"


def __getattr__(name):
    if name in __all__:
        return getattr(importlib.import_module(".kernels", __name__), name)
    if name in ("kernels", "tp", "synth", "weights", "_lib"):
        return importlib.import_module("." + name, __name__)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
