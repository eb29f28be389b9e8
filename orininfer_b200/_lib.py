"""ctypes binding of liborin_b200.so (the C ABI declared in include/orin_b200.h).

The library is built in-tree by ``python -m orininfer_b200.build``.  There is
no fallback: if the library is missing or fails to load, importing this module
raises, so no caller can silently run anything but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liborin_b200.so"

# orin_status
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_NCCL = 4
ERR_TIMEOUT = 5
ERR_NO_DEVICE = 6
STATUS_NAMES = {
    OK: "ORIN_OK", ERR_INVALID_ARG: "ORIN_ERR_INVALID_ARG", ERR_UNSUPPORTED: "ORIN_ERR_UNSUPPORTED",
    ERR_CUDA: "ORIN_ERR_CUDA", ERR_NCCL: "ORIN_ERR_NCCL", ERR_TIMEOUT: "ORIN_ERR_TIMEOUT",
    ERR_NO_DEVICE: "ORIN_ERR_NO_DEVICE",
}

# orin_dtype
F16 = 0
BF16 = 1

# orin_epilogue
EPI_NONE = 0
EPI_SWIGLU = 1
EPI_RESIDUAL = 2
EPI_F32_OUT = 3
EPI_F32_PARTIAL = 4

# orin_algo
ALGO_AUTO = 0
ALGO_TC_WIDE = 1
ALGO_TC_SKINNY = 2
ALGO_SIMT = 3
ALGO_GEMV = 4

TP_UNIQUE_ID_BYTES = 128

_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/orin_b200.h declares
SIGNATURES = {
    "orin_version": (_i, []),
    "orin_last_error": (ctypes.c_char_p, []),
    "orin_linear": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "orin_linear_ex": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i, _vp]),
    "orin_lm_head_argmax": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "orin_linear_rmsnorm": (_i, [_vp, _vp, _vp, _vp, ctypes.c_float, _i, _i, _i, _i, _i, _vp]),
    "orin_lm_head_argmax_rmsnorm": (_i, [_vp, _vp, _vp, _vp, ctypes.c_float, _i, _i, _i, _i, _vp,
                                         _vp]),
    "orin_pack_gate_up": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "orin_plan_info": (_i, [_i, _i, _i, _i, _i, _i, ctypes.POINTER(_i)]),
    "orin_plan_info_ws": (_i, [_i, _i, _i, _i, _i, _i, _sz, ctypes.POINTER(_i)]),
    "orin_linear_ws": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp]),
    "orin_linear_workspace_bytes": (_i, [ctypes.POINTER(_sz)]),
    "orin_silu_mul": (_i, [_vp, _vp, _vp, _ll, _i, _vp]),
    "orin_add": (_i, [_vp, _vp, _ll, _i, _vp]),
    "orin_widen_f32": (_i, [_vp, _vp, _ll, _i, _vp]),
    "orin_kv_append": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "orin_embedding": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "orin_rmsnorm": (_i, [_vp, _vp, _vp, _i, _i, ctypes.c_float, _i, _vp]),
    "orin_rope": (_i, [_vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float, _i, _vp]),
    "orin_qkv_rope_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                  ctypes.c_float, ctypes.c_float, _i, _i, _i, _vp]),
    "orin_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float, _i, _i, _i,
                            _vp, _sz, _vp]),
    "orin_attention_workspace_bytes": (_i, [ctypes.POINTER(_sz), _i, _i, _i, _i, _i, _i, _i]),
    "orin_attention_batch": (_i, [_vp, _vp, _vp, _vp, _i, _ll, _i, _i, _i, _i, _i,
                                  ctypes.c_float, _i, _i, _i, _vp, _sz, _vp]),
    "orin_attention_batch_ex": (_i, [_vp, _vp, _vp, _vp, _i, _ll, _i, _i, _i, _i, _i,
                                     ctypes.c_float, _i, _i, _i, _vp, _sz, ctypes.c_uint, _vp]),
    "orin_qkv_rope_append_batch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _ll, _i, _i, _i, _i,
                                        _i, ctypes.c_float, ctypes.c_float, _i, _i, _i, _vp]),
    "orin_linear_rope_append": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _ll, _i, _i, _i, _i, _i, _i,
                                     ctypes.c_float, _i, _i, _i, _vp]),
    "orin_device_check": (_i, [_vp]),
    "orin_tp_unique_id": (_i, [_vp]),
    "orin_tp_init": (_i, [ctypes.POINTER(_vp), _vp, _i, _i, _i, ctypes.c_double]),
    "orin_tp_allreduce_f32": (_i, [_vp, _vp, _ll, _vp]),
    "orin_tp_linear_row": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "orin_tp_linear_row_static": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "orin_tp_static_partial_capacity": (_ll, []),
    "orin_tp_enable_p2p": (_i, [_vp, _ll, _vp]),
    "orin_p2p_watchdog_selftest": (_i, [_vp]),
    "orin_tp_lm_head_argmax": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "orin_tp_wait": (_i, [_vp, _vp]),
    "orin_tp_destroy": (_i, [_vp]),
}

# C++ entry points with the reference's exact signatures (include/orin_kernels.h)
SHIM_SYMBOLS = {
    "kernels::matmul": "_ZN7kernels6matmulEP13__nv_bfloat16PKS0_S3_iii",
    "kernels::fused_silu_mul": "_ZN7kernels14fused_silu_mulEP13__nv_bfloat16PKS0_S3_ii",
    "kernels::add": "_ZN7kernels3addEP13__nv_bfloat16PKS0_i",
    "kernels::bf16_to_fp32": "_ZN7kernels12bf16_to_fp32EPfPK13__nv_bfloat16i",
    "launch_gemm_cute": "_Z16launch_gemm_cuteP13__nv_bfloat16PKS_S2_iii",
    "kernels::attention": "_ZN7kernels9attentionEP13__nv_bfloat16PKS0_S3_S3_iiiiifii",
    "kernels::rmsnorm": "_ZN7kernels7rmsnormEP13__nv_bfloat16PKS0_S3_iif",
    "kernels::embedding": "_ZN7kernels9embeddingEP13__nv_bfloat16PKS0_PKiii",
    "kernels::rope": "_ZN7kernels4ropeEP13__nv_bfloat16S1_iiiiif",
}


class OrinError(RuntimeError):
    """A non-OK orin_status, with the library's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m orininfer_b200.build` "
            "(there is no CPU fallback)")
    # RTLD_LOCAL: the library's C++ drop-in symbols (kernels::matmul, ...) must
    # not become the global definitions other libraries in this process bind to
    lib = ctypes.CDLL(os.fspath(LIB_PATH), mode=os.RTLD_LOCAL | os.RTLD_NOW)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    shim_args = {
        "kernels::matmul": [_vp, _vp, _vp, _i, _i, _i],
        "kernels::fused_silu_mul": [_vp, _vp, _vp, _i, _i],
        "kernels::add": [_vp, _vp, _i],
        "kernels::bf16_to_fp32": [_vp, _vp, _i],
        "launch_gemm_cute": [_vp, _vp, _vp, _i, _i, _i],
        "kernels::attention": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float, _i, _i],
        "kernels::rmsnorm": [_vp, _vp, _vp, _i, _i, ctypes.c_float],
        "kernels::embedding": [_vp, _vp, _vp, _i, _i],
        "kernels::rope": [_vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float],
    }
    for name, sym in SHIM_SYMBOLS.items():
        fn = getattr(lib, sym)
        fn.restype = ctypes.c_bool if name == "launch_gemm_cute" else None
        fn.argtypes = shim_args[name]
    return lib


lib = _load()


def check(status: int) -> None:
    """Raise OrinError for a non-OK status."""
    if status != OK:
        msg = lib.orin_last_error()
        raise OrinError(status, msg.decode() if msg else "")


def shim(name: str):
    """The C++ drop-in entry point `name` (e.g. "kernels::matmul")."""
    return getattr(lib, SHIM_SYMBOLS[name])
