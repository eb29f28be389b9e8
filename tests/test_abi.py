"""The C ABI library: loads, exports every declared entry point, rejects bad
arguments on the host before any device work (CPU only)."""
import ctypes
import os
import re

import pytest
import torch

from orininfer_b200 import _lib
from orininfer_b200 import kernels as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_c_symbols():
    src = open(os.path.join(ROOT, "include", "orin_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(orin_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    names = declared_c_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} declared in include/orin_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_library_exports_reference_cxx_entry_points():
    hdr = open(os.path.join(ROOT, "include", "orin_kernels.h")).read()
    for name in ("matmul", "fused_silu_mul", "add", "bf16_to_fp32", "launch_gemm_cute",
                 "attention", "rmsnorm", "rope", "embedding"):
        assert re.search(rf"\b{name}\s*\(", hdr)
    for name, sym in _lib.SHIM_SYMBOLS.items():
        assert hasattr(_lib.lib, sym), f"{name} ({sym}) not exported"


def test_version():
    assert _lib.lib.orin_version() >= 100


@pytest.mark.parametrize("kw,code", [
    (dict(dtype=7), _lib.ERR_INVALID_ARG),
    (dict(epi=9), _lib.ERR_INVALID_ARG),
    (dict(M=0), _lib.ERR_INVALID_ARG),
    (dict(N=-1), _lib.ERR_INVALID_ARG),
    (dict(K=0), _lib.ERR_INVALID_ARG),
    (dict(C=0), _lib.ERR_INVALID_ARG),
    (dict(epi=_lib.EPI_RESIDUAL, R=0), _lib.ERR_INVALID_ARG),
    (dict(epi=_lib.EPI_SWIGLU, N=100), _lib.ERR_UNSUPPORTED),
    (dict(algo=9), _lib.ERR_INVALID_ARG),
])
def test_linear_rejects_bad_arguments_on_host(kw, code):
    a = dict(C=16, A=32, W=48, M=4, N=128, K=64, dtype=_lib.F16, epi=_lib.EPI_NONE, R=0, algo=0)
    a.update(kw)
    st = _lib.lib.orin_linear_ex(a["C"], a["A"], a["W"], a["M"], a["N"], a["K"], a["dtype"],
                                 a["epi"], a["R"], a["algo"], None)
    assert st == code
    assert _lib.lib.orin_last_error()


def test_skinny_algo_rejects_wide_m():
    st = _lib.lib.orin_linear_ex(16, 32, 48, 65, 128, 64, _lib.F16, 0, 0, _lib.ALGO_TC_SKINNY,
                                 None)
    assert st == _lib.ERR_UNSUPPORTED


def test_tc_algo_rejects_unaligned_k():
    st = _lib.lib.orin_linear_ex(16, 32, 48, 4, 128, 12, _lib.F16, 0, 0, _lib.ALGO_TC_WIDE,
                                 None)
    assert st == _lib.ERR_UNSUPPORTED


def test_elementwise_and_pack_reject_bad_arguments():
    L = _lib.lib
    assert L.orin_silu_mul(None, None, None, -1, 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_add(None, 16, 10, 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_widen_f32(16, 16, 10, 5, None) == _lib.ERR_INVALID_ARG
    assert L.orin_pack_gate_up(16, 16, 16, 100, 64, 0, None) == _lib.ERR_UNSUPPORTED
    assert L.orin_pack_gate_up(None, 16, 16, 128, 64, 0, None) == _lib.ERR_INVALID_ARG
    # zero-length elementwise calls are no-ops
    assert L.orin_add(None, None, 0, 0, None) == _lib.OK


def test_tp_rejects_bad_arguments():
    L = _lib.lib
    h = ctypes.c_void_p()
    assert L.orin_tp_init(ctypes.byref(h), None, 0, 1, 0, 1.0) == _lib.ERR_INVALID_ARG
    buf = ctypes.create_string_buffer(128)
    assert L.orin_tp_init(ctypes.byref(h), buf, 2, 2, 0, 1.0) == _lib.ERR_INVALID_ARG
    assert L.orin_tp_allreduce_f32(None, 16, 4, None) == _lib.ERR_INVALID_ARG
    assert L.orin_tp_linear_row(None, 16, 16, 16, 1, 1, 1, 0, None, None, None) == _lib.ERR_INVALID_ARG
    assert L.orin_tp_destroy(None) == _lib.OK
    assert L.orin_tp_enable_p2p(None, 1 << 20, None) == _lib.ERR_INVALID_ARG
    assert L.orin_tp_lm_head_argmax(None, 16, 16, 16, 1, 10, 0, 64, 0, 16, None) == \
        _lib.ERR_INVALID_ARG
    dummy = ctypes.c_void_p(16)
    assert L.orin_tp_enable_p2p(dummy, 4, None) == _lib.ERR_INVALID_ARG         # < 8 elements
    assert L.orin_tp_lm_head_argmax(dummy, 16, 16, 16, 1, 10, -1, 64, 0, 16, None) == \
        _lib.ERR_INVALID_ARG                                                    # negative offset


def test_lm_head_argmax_rejects_bad_arguments_on_host():
    L = _lib.lib
    assert L.orin_lm_head_argmax(None, 16, 16, 1, 10, 64, 0, 16, None) == _lib.ERR_INVALID_ARG
    assert L.orin_lm_head_argmax(16, 16, 16, 0, 10, 64, 0, 16, None) == _lib.ERR_INVALID_ARG
    assert L.orin_lm_head_argmax(16, 16, 16, 1, 10, 64, 7, 16, None) == _lib.ERR_INVALID_ARG
    # K % 8 != 0: the weight stream can't take it
    assert L.orin_lm_head_argmax(16, 16, 16, 1, 10, 12, 0, 16, None) == _lib.ERR_UNSUPPORTED
    # unaligned h
    assert L.orin_lm_head_argmax(16, 18, 16, 1, 10, 64, 0, 16, None) == _lib.ERR_UNSUPPORTED


def test_python_mirror_rejects_cpu_tensors():
    x = torch.zeros(4, 64, dtype=torch.float16)
    w = torch.zeros(128, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        K.linear(x, w)
    with pytest.raises(ValueError):
        K.matmul(torch.zeros(4, 128, dtype=torch.float16), x, w, 4, 128, 64)


def test_attention_and_kv_append_reject_bad_arguments_on_host():
    L = _lib.lib
    f = ctypes.c_float(0.125)
    ok = dict(out=16, q=16, k=16, v=16, S=1, C=10, nh=32, nkv=4, hd=64, ns=4, W=1024, dt=0)

    def att(**kw):
        a = dict(ok, **kw)
        return L.orin_attention(a["out"], a["q"], a["k"], a["v"], a["S"], a["C"], a["nh"],
                                a["nkv"], a["hd"], f, a["ns"], a["W"], a["dt"], None, 0, None)

    assert att(nkv=5) == _lib.ERR_INVALID_ARG        # heads not a multiple of kv heads
    assert att(C=0) == _lib.ERR_INVALID_ARG          # cache_len < seq_len
    assert att(W=0) == _lib.ERR_INVALID_ARG
    assert att(ns=-1) == _lib.ERR_INVALID_ARG
    assert att(dt=3) == _lib.ERR_INVALID_ARG
    assert att(q=0) == _lib.ERR_INVALID_ARG
    assert att(hd=96) == _lib.ERR_UNSUPPORTED
    assert att(k=24) == _lib.ERR_UNSUPPORTED         # pool not 16-byte aligned
    assert att(S=0, C=0, out=0) == _lib.OK           # nothing to do
    assert L.orin_kv_append(16, 16, 16, 16, 1029, 0, 4, 1024, 256, 0, None) == \
        _lib.ERR_INVALID_ARG                          # seq_len > n_sink + window (reference throws)
    assert L.orin_kv_append(0, 16, 16, 16, 4, 0, 4, 1024, 256, 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_kv_append(16, 16, 16, 16, 4, -1, 4, 1024, 256, 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_kv_append(16, 16, 16, 16, 0, 0, 4, 1024, 256, 0, None) == _lib.OK


def test_batched_attention_and_append_reject_bad_arguments_on_host():
    """The batched decode entry points check the pool stride (at least one
    pool apart) and the single-sequence arguments before any device work."""
    L = _lib.lib
    f = ctypes.c_float(0.125)
    pool = (4 + 1024) * 4 * 64

    def att(batch=2, stride=pool, **kw):
        a = dict(dict(out=16, q=16, k=16, v=16, S=1, C=10, nh=32, nkv=4, hd=64, ns=4, W=1024,
                      dt=0), **kw)
        return L.orin_attention_batch(a["out"], a["q"], a["k"], a["v"], batch, stride, a["S"],
                                      a["C"], a["nh"], a["nkv"], a["hd"], f, a["ns"], a["W"],
                                      a["dt"], None, 0, None)

    assert att(stride=pool - 8) == _lib.ERR_INVALID_ARG     # pools would overlap
    assert att(batch=-1) == _lib.ERR_INVALID_ARG
    assert att(nkv=5) == _lib.ERR_INVALID_ARG
    assert att(stride=pool + 4) == _lib.ERR_UNSUPPORTED     # stride not 16-byte aligned
    assert att(batch=20000) == _lib.ERR_UNSUPPORTED         # grid y above 65535
    assert att(batch=0) == _lib.OK
    # the flags form: unknown flags are refused before anything else
    assert L.orin_attention_batch_ex(16, 16, 16, 16, 2, pool, 1, 10, 32, 4, 64, f, 4, 1024, 0,
                                     None, 0, 2, None) == _lib.ERR_INVALID_ARG
    assert L.orin_attention_batch_ex(16, 16, 16, 16, 0, pool, 1, 10, 32, 4, 64, f, 4, 1024, 0,
                                     None, 0, 1, None) == _lib.OK

    def app(batch=2, stride=pool, S=1, start=7, q_out=16):
        return L.orin_qkv_rope_append_batch(q_out, 16, None, None, 16, 16, batch, stride, S,
                                            start, 32, 4, 64, ctypes.c_float(1e-5),
                                            ctypes.c_float(1e4), 4, 1024, 0, None)

    assert app(stride=pool - 1) == _lib.ERR_INVALID_ARG
    assert app(S=1029) == _lib.ERR_INVALID_ARG              # more than n_sink + window
    assert app(start=-1) == _lib.ERR_INVALID_ARG
    assert app(q_out=0) == _lib.ERR_INVALID_ARG
    assert app(batch=0) == _lib.OK

    def lra(batch=2, stride=pool, S=1, start=7, hidden=2048, hd=64, x=16, nkv=4):
        return L.orin_linear_rope_append(16, x, 16, 16, 16, batch, stride, S, start, hidden, 32,
                                         nkv, hd, ctypes.c_float(1e4), 4, 1024, 0, None)

    # every rejection comes before any device work
    assert lra(stride=pool - 1) == _lib.ERR_INVALID_ARG     # pools would overlap
    assert lra(batch=0) == _lib.ERR_INVALID_ARG
    assert lra(S=1029) == _lib.ERR_INVALID_ARG              # more than n_sink + window
    assert lra(start=-1) == _lib.ERR_INVALID_ARG
    assert lra(nkv=5) == _lib.ERR_INVALID_ARG
    assert lra(x=0) == _lib.ERR_INVALID_ARG
    assert lra(batch=33, stride=pool) == _lib.ERR_UNSUPPORTED  # more than 32 token rows
    assert lra(hidden=2044) == _lib.ERR_UNSUPPORTED         # hidden % 8
    assert lra(x=24) == _lib.ERR_UNSUPPORTED                # x not 16-byte aligned
    assert lra(hd=96, stride=(4 + 1024) * 4 * 96) == _lib.ERR_UNSUPPORTED  # 64 and 128 built


def test_attention_workspace_plan():
    """Few-token calls split their keys across CTAs; prefill-sized calls don't.
    The split count for TinyLlama decode (32 heads over 4 KV heads, window
    1024 + 4 sinks) is one per 64-key tile: 17.  A split workspace holds 4 KB
    of arrival counters, then the partials (O, running max and sum per row)."""
    ws = K.attention_workspace_bytes
    counters = 4096
    assert ws(1, 2048, 32, 4, 64, 4, 1024) == counters + 17 * 32 * (64 + 2) * 4
    assert ws(1, 3, 32, 4, 64, 4, 1024) == 0            # one key tile: nothing to split
    assert ws(1028, 1028, 32, 4, 64, 4, 1024) == 0      # 516 CTAs without splitting
    assert ws(1, 3000, 32, 8, 128, 4, 1024) == counters + 17 * 32 * (128 + 2) * 4
    assert ws(0, 0, 32, 4, 64, 4, 1024) == 0


def test_attention_split_cap_override():
    """ORIN_ATTN_SPLITS (a tuning override, read once per process) caps the
    key splits of decode row blocks: the plan's workspace shrinks with it;
    prefill-sized calls are untouched."""
    import os
    import subprocess
    import sys
    code = ("from orininfer_b200 import kernels as K; "
            "print(K.attention_workspace_bytes(1, 2048, 32, 4, 64, 4, 1024), "
            "K.attention_workspace_bytes(1028, 1028, 32, 4, 64, 4, 1024))")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, ORIN_ATTN_SPLITS="4", PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=root, capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    decode, prefill = (int(v) for v in r.stdout.split())
    assert decode == 4096 + 4 * 32 * (64 + 2) * 4
    assert prefill == 0


def test_norm_and_rope_reject_bad_arguments_on_host():
    L = _lib.lib
    f = ctypes.c_float
    assert L.orin_embedding(16, 16, 16, 1, 64, 0, None) == _lib.ERR_INVALID_ARG    # no vocab
    assert L.orin_embedding(None, 16, 16, 1, 64, 10, None) == _lib.ERR_INVALID_ARG
    assert L.orin_embedding(16, 16, 16, 0, 64, 10, None) == _lib.OK
    assert L.orin_rmsnorm(16, 16, 16, 1, 0, f(1e-5), 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_rmsnorm(None, 16, 16, 1, 64, f(1e-5), 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_rmsnorm(16, 16, 16, 0, 64, f(1e-5), 0, None) == _lib.OK
    assert L.orin_rope(16, 16, 1, 4, 2, 63, 0, f(1e4), 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_rope(16, 16, 1, 4, 2, 64, -1, f(1e4), 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_rope(None, 16, 1, 4, 2, 64, 0, f(1e4), 0, None) == _lib.ERR_INVALID_ARG

    def fused(**kw):
        a = dict(qo=16, qkv=16, qn=0, kn=0, kp=16, vp=16, S=1, pos=0, nh=32, nkv=4, hd=64,
                 ns=4, W=1024, dt=0)
        a.update(kw)
        return L.orin_qkv_rope_append(a["qo"], a["qkv"], a["qn"], a["kn"], a["kp"], a["vp"],
                                      a["S"], a["pos"], a["nh"], a["nkv"], a["hd"], f(1e-6),
                                      f(1e4), a["ns"], a["W"], a["dt"], None)

    assert fused(qn=16) == _lib.ERR_INVALID_ARG       # q_norm without k_norm
    assert fused(nkv=5) == _lib.ERR_INVALID_ARG
    assert fused(S=1029) == _lib.ERR_INVALID_ARG      # more than n_sink + window
    assert fused(hd=96) == _lib.ERR_UNSUPPORTED
    assert fused(S=0) == _lib.OK


def test_folded_norm_entry_points_reject_bad_arguments_on_host():
    L = _lib.lib
    f = ctypes.c_float(1e-5)
    # C, A, W, norm, eps, M, N, K, dtype, epilogue
    assert L.orin_linear_rmsnorm(16, 16, 16, 0, f, 1, 64, 64, 0, 0, None) == _lib.ERR_INVALID_ARG
    assert L.orin_linear_rmsnorm(16, 16, 16, 16, f, 33, 64, 64, 0, 0, None) == \
        _lib.ERR_UNSUPPORTED                                   # more tokens than the stream takes
    assert L.orin_linear_rmsnorm(16, 16, 16, 16, f, 1, 64, 60, 0, 0, None) == \
        _lib.ERR_UNSUPPORTED                                   # K % 8 != 0
    assert L.orin_linear_rmsnorm(16, 16, 16, 16, f, 1, 64, 64, 0, 2, None) == \
        _lib.ERR_UNSUPPORTED                                   # residual does not follow a norm
    assert L.orin_linear_rmsnorm(16, 16, 16, 16, f, 1, 100, 64, 0, 1, None) == \
        _lib.ERR_UNSUPPORTED                                   # SwiGLU needs N % 64 == 0
    assert L.orin_lm_head_argmax_rmsnorm(16, 16, 16, 0, f, 1, 10, 64, 0, 16, None) == \
        _lib.ERR_INVALID_ARG
    assert L.orin_lm_head_argmax_rmsnorm(16, 16, 16, 24, f, 1, 10, 64, 0, 16, None) == \
        _lib.ERR_UNSUPPORTED                                   # unaligned norm weight
