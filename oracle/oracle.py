"""Python binding of the oracle (oracle/liborc.so) and of the reference's own
kernels compiled from its sources (oracle/_ref/*.so).

TEST INFRASTRUCTURE ONLY: the tests, the smoke check and the bench's CPU
baseline use this module as the checker; nothing in orininfer_b200 imports it.

Arrays are numpy uint16 holding 16-bit float bit patterns (fp16 or bf16).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liborc.so"
REF_CUBLAS = HERE / "_ref" / "libref_cublas.so"
REF_CUTE = HERE / "_ref" / "libref_cute.so"

F16, BF16 = 0, 1
EPI = {"none": 0, "swiglu": 1, "residual": 2, "f32": 3, "f32_partial": 4}

_vp, _i, _ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong


def reference_tree() -> Path | None:
    """The reference source tree the checkers are compiled from: $ORIN_REFERENCE_TREE,
    else the Makefile's default REF; None where it is absent (a machine that only
    runs the prebuilt files)."""
    ref = Path(os.environ.get("ORIN_REFERENCE_TREE", "/root/reference"))
    return ref if (ref / "kernels" / "matmul.cu").exists() else None


def build() -> None:
    """Compile liborc.so (and the reference checkers when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", os.fspath(HERE), "orc"], check=True)
    ref = reference_tree()
    if ref is not None:
        subprocess.run(["make", "-s", "-C", os.fspath(HERE), f"REF={ref}", "ref"], check=True)


def _load() -> ctypes.CDLL:
    if not LIB.exists():
        build()
    lib = ctypes.CDLL(os.fspath(LIB))
    lib.orc_linear.restype = _i
    lib.orc_linear.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i]
    lib.orc_gemm_f32.restype = None
    lib.orc_gemm_f32.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i]
    for n in ("orc_silu_mul",):
        getattr(lib, n).argtypes = [_vp, _vp, _vp, _ll, _i]
    lib.orc_add.argtypes = [_vp, _vp, _ll, _i]
    lib.orc_widen.argtypes = [_vp, _vp, _ll, _i]
    lib.orc_round.argtypes = [_vp, _vp, _ll, _i]
    lib.orc_pack_gate_up.argtypes = [_vp, _vp, _vp, _i, _i]
    lib.orc_max_threads.restype = _i
    lib.orc_gemv_reference_order.argtypes = [_vp, _vp, _vp, _i, _i, _i]
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _p(a: np.ndarray | None) -> ctypes.c_void_p:
    if a is None:
        return ctypes.c_void_p(0)
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


def max_threads() -> int:
    return int(lib().orc_max_threads())


def linear(A: np.ndarray, W: np.ndarray, dt: int, epilogue: str = "none",
           R: np.ndarray | None = None, threads: int = 0) -> np.ndarray:
    """epilogue(A · W^T) with the reference's rounding points (orc.c:orc_linear)."""
    A = np.ascontiguousarray(A, dtype=np.uint16)
    W = np.ascontiguousarray(W, dtype=np.uint16)
    M, K = A.shape
    N = W.shape[0] // 2 if epilogue == "swiglu" else W.shape[0]
    if epilogue in ("f32", "f32_partial"):
        C = np.empty((M, N), dtype=np.float32)
    else:
        C = np.empty((M, N), dtype=np.uint16)
    if R is not None:
        R = np.ascontiguousarray(R, dtype=np.uint16)
    rc = lib().orc_linear(_p(C), _p(A), _p(W), M, N, K, dt, EPI[epilogue], _p(R), threads)
    if rc != 0:
        raise MemoryError("orc_linear: allocation failed")
    return C


def gemv_reference_order(A: np.ndarray, B: np.ndarray, dt: int) -> np.ndarray:
    """The reference GEMV's own summation order (orc.c:orc_gemv_reference_order)."""
    A = np.ascontiguousarray(A, dtype=np.uint16).reshape(-1)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    N, K = B.shape
    C = np.empty((1, N), dtype=np.uint16)
    lib().orc_gemv_reference_order(_p(C), _p(A), _p(B), N, K, dt)
    return C


def gemm_f32(A: np.ndarray, W: np.ndarray, threads: int = 0) -> np.ndarray:
    """Multithreaded fp32 C = A · W^T (the CPU baseline)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    C = np.empty((A.shape[0], W.shape[0]), dtype=np.float32)
    lib().orc_gemm_f32(_p(A), _p(W), _p(C), A.shape[0], W.shape[0], A.shape[1], threads)
    return C


def silu_mul(g: np.ndarray, u: np.ndarray, dt: int) -> np.ndarray:
    out = np.empty_like(g, dtype=np.uint16)
    lib().orc_silu_mul(_p(out), _p(np.ascontiguousarray(g)), _p(np.ascontiguousarray(u)),
                       g.size, dt)
    return out


def add(x: np.ndarray, y: np.ndarray, dt: int) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.uint16).copy()
    lib().orc_add(_p(out), _p(np.ascontiguousarray(y)), out.size, dt)
    return out


def widen(x: np.ndarray, dt: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty(x.shape, dtype=np.float32)
    lib().orc_widen(_p(x), _p(out), x.size, dt)
    return out


def round16(x: np.ndarray, dt: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_round(_p(x), _p(out), x.size, dt)
    return out


def argmax_reference(x: np.ndarray, threads: int = 512) -> int:
    """The reference's greedy sampler (kernels/softmax.cu:52-73, launched with
    512 threads at :108-110), restated step by step: thread t scans
    i = t, t+512, ... keeping the first strictly greater value (start -FLT_MAX,
    index 0), then a halving tree where slot t takes slot t+s only if strictly
    greater.  x: float32 logits of one row."""
    x = np.asarray(x, dtype=np.float32)
    neg = np.float32(-3.4028234663852886e38)
    val = np.full(threads, neg, dtype=np.float32)
    idx = np.zeros(threads, dtype=np.int64)
    for t in range(threads):
        for i in range(t, x.shape[0], threads):
            if x[i] > val[t]:
                val[t], idx[t] = x[i], i
    s = threads // 2
    while s > 0:
        for t in range(s):
            if val[t + s] > val[t]:
                val[t], idx[t] = val[t + s], idx[t + s]
        s //= 2
    return int(idx[0])


def argmax_key_order(x: np.ndarray) -> int:
    """The same choice as argmax_reference, stated as an order: among the
    positions of the maximum (values > -FLT_MAX only; none -> 0), the one whose
    residue i mod 512 has the smallest 9-bit bit-reversal (ties in the tree
    meet at their lowest differing bit, where the 0 side wins), then the
    smallest i.  This is the order the fused LM-head argmax packs into its
    64-bit keys."""
    x = np.asarray(x, dtype=np.float32)
    ok = x > np.float32(-3.4028234663852886e38)
    if not ok.any():
        return 0
    best = x[ok].max()
    cand = np.nonzero(ok & (x == best))[0]

    def rev9(t: int) -> int:
        return int(format(t, "09b")[::-1], 2)

    return int(min(cand, key=lambda i: (rev9(int(i) % 512), int(i))))


def lm_head_argmax(h: np.ndarray, W: np.ndarray, dt: int) -> np.ndarray:
    """Greedy next token per row of h: the LM head with the reference's
    rounding (16-bit logits widened to fp32, src/model.cu:125-130) followed by
    argmax_reference."""
    logits = linear(h, W, dt, "f32")
    return np.array([argmax_reference(row) for row in logits], dtype=np.int32)


def pack_gate_up(wg: np.ndarray, wu: np.ndarray) -> np.ndarray:
    wg = np.ascontiguousarray(wg, dtype=np.uint16)
    wu = np.ascontiguousarray(wu, dtype=np.uint16)
    IM, K = wg.shape
    out = np.empty((2 * IM, K), dtype=np.uint16)
    lib().orc_pack_gate_up(_p(out), _p(wg), _p(wu), IM, K)
    return out


def ring_slot(pos, n_sink: int, window: int):
    """Pool slot of logical position pos (src/kv_cache.cu:29-31)."""
    pos = np.asarray(pos, dtype=np.int64)
    return np.where(pos < n_sink, pos, n_sink + (pos - n_sink) % window)


def kv_append(k_pool: np.ndarray, v_pool: np.ndarray, k_src: np.ndarray, v_src: np.ndarray,
              start_pos: int, n_sink: int, window: int) -> None:
    """KVCache::append_kv (src/kv_cache.cu:95-111, kernel :21-41): row t of the
    call goes to the slot of position start_pos + t, in place; rows taken in
    call order, so of two rows sharing a slot the later one stays.
    Pools [slots, kv_dim], sources [seq_len, kv_dim] (any dtype)."""
    seq_len = k_src.shape[0]
    if seq_len > n_sink + window:
        raise ValueError("seq_len exceeds n_sink + window (src/kv_cache.cu:99-103)")
    slots = ring_slot(start_pos + np.arange(seq_len), n_sink, window)
    for t in range(seq_len):
        k_pool[slots[t]] = k_src[t]
        v_pool[slots[t]] = v_src[t]


def attention(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, seq_len: int,
              cache_len: int, num_heads: int, num_kv_heads: int, head_dim: int, scale: float,
              n_sink: int, window: int, dt: int) -> np.ndarray:
    """Sink + sliding-window GQA attention (kernels/attention.cu:27-138), vectorised.

    q: uint16 bits [seq_len, num_heads, head_dim]; pools: uint16 bits
    [n_sink + window, num_kv_heads, head_dim]; returns uint16 bits of out
    [seq_len, num_heads, head_dim].  Query token t (attend_pos
    ap = cache_len - seq_len + t, :47) sees positions p <= ap with p < n_sink
    (the sink, :48) or p >= ap + 1 - window (the window, :49-55), each read
    from its ring slot; scores scale * q.k (:66-82), softmax (:87-118) and the
    weighted sum of V (:121-137) in float64 here (fp32 in the reference), one
    rounding of the result to the 16-bit type (:137)."""
    G = num_heads // num_kv_heads
    qf = widen(q, dt).reshape(seq_len, num_heads, head_dim).astype(np.float64)
    kf = widen(k_pool, dt).reshape(-1, num_kv_heads, head_dim).astype(np.float64)
    vf = widen(v_pool, dt).reshape(-1, num_kv_heads, head_dim).astype(np.float64)
    ap = cache_len - seq_len + np.arange(seq_len)
    sink_hi = min(n_sink, int(ap[-1]) + 1)
    win_lo = max(n_sink, int(ap[0]) + 1 - window)
    pos = np.concatenate([np.arange(sink_hi), np.arange(win_lo, int(ap[-1]) + 1)])
    slot = ring_slot(pos, n_sink, window)
    ok = (pos[None, :] <= ap[:, None]) & (
        (pos[None, :] < n_sink) | (pos[None, :] >= ap[:, None] + 1 - window))
    out = np.empty((seq_len, num_heads, head_dim), dtype=np.float64)
    for h in range(num_kv_heads):
        K = kf[slot, h]  # [U, hd]
        V = vf[slot, h]
        Q = qf[:, h * G:(h + 1) * G]  # [seq, G, hd]
        s = np.einsum("tgd,ud->tgu", Q, K) * scale
        s = np.where(ok[:, None, :], s, -np.inf)
        m = s.max(axis=-1, keepdims=True)
        e = np.exp(s - m)
        out[:, h * G:(h + 1) * G] = np.einsum("tgu,ud->tgd", e, V) / e.sum(axis=-1)[..., None]
    return round16(out.astype(np.float32), dt)


def attention_literal(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, seq_len: int,
                      cache_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                      scale: float, n_sink: int, window: int, dt: int) -> np.ndarray:
    """The same, step by step as one CTA of kernels/attention.cu:27-138 runs it
    (small cases only): sink_len, window_len, the oldest window position and
    the ring offset win_offset, physical slot n_sink + (win_offset + w) %
    window of the w-th window token; fp32 scores, max, exp, sum and the
    normalised weighted sum of V."""
    G = num_heads // num_kv_heads
    qf = widen(q, dt).reshape(seq_len, num_heads, head_dim)
    kf = widen(k_pool, dt).reshape(-1, num_kv_heads, head_dim)
    vf = widen(v_pool, dt).reshape(-1, num_kv_heads, head_dim)
    out = np.empty((seq_len, num_heads, head_dim), dtype=np.float32)
    f32 = np.float32
    for qi in range(seq_len):
        for h in range(num_heads):
            kv_h = h // G
            attend_pos = cache_len - seq_len + qi
            sink_len = min(n_sink, attend_pos + 1)
            window_len = min(max(attend_pos + 1 - n_sink, 0), window)
            oldest_w = attend_pos + 1 - window_len
            win_offset = (oldest_w - n_sink) % window if window_len > 0 else 0
            phys = list(range(sink_len)) + [n_sink + (win_offset + w) % window
                                            for w in range(window_len)]
            scores = np.array([f32(np.dot(qf[qi, h], kf[ph, kv_h])) * f32(scale) for ph in phys],
                              dtype=np.float32)
            e = np.exp(scores - scores.max()).astype(np.float32)
            p = e * (f32(1.0) / e.sum(dtype=np.float32))
            out[qi, h] = (p[:, None] * vf[phys, kv_h]).sum(axis=0, dtype=np.float32)
    return round16(out, dt)


def rmsnorm(x: np.ndarray, w: np.ndarray, dt: int, eps: float) -> np.ndarray:
    """kernels/rmsnorm.cu:7-34 per row of the last axis: r = rsqrt(sum(x^2) / dim
    + eps) in fp32 (the sum in float64 here), out = round16(x * r * w) in fp32."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    xf = widen(x, dt)
    wf = widen(np.ascontiguousarray(w, dtype=np.uint16), dt)
    dim = x.shape[-1]
    ss = (xf.astype(np.float64) ** 2).sum(axis=-1).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(ss / np.float32(dim) + np.float32(eps))).astype(np.float32)
    return round16((xf * r[..., None]) * wf, dt)


def rope(x: np.ndarray, start_pos: int, theta: float, dt: int) -> np.ndarray:
    """kernels/rope.cu:7-37 on x [seq, heads, head_dim] (bits): pair (i, i + hd/2)
    of token t rotates by (start_pos + t) * theta^(-2i/hd), fp32 angle, each
    result rounded to 16 bits."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    seq, heads, hd = x.shape
    half = hd // 2
    xf = widen(x, dt)
    i = np.arange(half, dtype=np.float32)
    inv = np.power(np.float32(theta), (np.float32(-2.0) * i) / np.float32(hd)).astype(np.float32)
    pos = (start_pos + np.arange(seq)).astype(np.float32)
    ang = (pos[:, None] * inv[None, :]).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    sn = np.sin(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    x0, x1 = xf[..., :half], xf[..., half:]
    out = np.empty_like(x)
    out[..., :half] = round16(x0 * c - x1 * sn, dt)
    out[..., half:] = round16(x0 * sn + x1 * c, dt)
    return out


def transformer_layer(x: np.ndarray, L: dict, k_pool: np.ndarray, v_pool: np.ndarray,
                      start_pos: int, cfg: dict, dt: int) -> np.ndarray:
    """Model::transformer_layer (src/model.cu:37-111) on seq_len = len(x) tokens:
    x [seq, H] bits -> new x; the pools [n_sink + W, kv_dim] bits are appended
    in place.  L holds bits of input_layernorm, q/k/v/o_proj, post_attention_layernorm,
    gate/up/down_proj and, for Qwen3, q_norm / k_norm (absent: Llama, no
    q/k norm).  cfg: num_attention_heads, num_key_value_heads, head_dim,
    rms_norm_eps, rope_theta, n_sink, window."""
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    eps, theta = cfg["rms_norm_eps"], cfg["rope_theta"]
    ns, W = cfg["n_sink"], cfg["window"]
    seq = x.shape[0]
    xn = rmsnorm(x, L["input_layernorm"], dt, eps)                        # :53
    q = linear(xn, L["q_proj"], dt)                                       # :59-61
    k = linear(xn, L["k_proj"], dt)
    v = linear(xn, L["v_proj"], dt)
    if L.get("q_norm") is not None:                                       # :64-67
        q = rmsnorm(q.reshape(-1, hd), L["q_norm"], dt, eps)
        k = rmsnorm(k.reshape(-1, hd), L["k_norm"], dt, eps)
    q = rope(q.reshape(seq, nh, hd), start_pos, theta, dt)                # :70-73
    k = rope(k.reshape(seq, nkv, hd), start_pos, theta, dt)
    kv_append(k_pool, v_pool, k.reshape(seq, nkv * hd), v.reshape(seq, nkv * hd),
              start_pos, ns, W)                                           # :75
    att = attention(q, k_pool.reshape(-1, nkv, hd), v_pool.reshape(-1, nkv, hd), seq,
                    start_pos + seq, nh, nkv, hd, float(np.float32(1.0) / np.sqrt(np.float32(hd))),
                    ns, W, dt)                                            # :79-84
    o = linear(att.reshape(seq, nh * hd), L["o_proj"], dt)                # :87
    x = add(x, o, dt)                                                     # :90
    xn = rmsnorm(x, L["post_attention_layernorm"], dt, eps)               # :95
    g = linear(xn, L["gate_proj"], dt)                                    # :100-101
    u = linear(xn, L["up_proj"], dt)
    h = silu_mul(g, u, dt)                                                # :104
    d = linear(h, L["down_proj"], dt)                                     # :107
    return add(x, d, dt)                                                  # :110


REF_REFUSED_CUTE = -2  # ref_entry.cu: the call would have reached the CuTe kernel


def cute_refused(M: int, N: int, K: int) -> bool:
    """True for the shapes that the reference's build without cuBLAS sends to its
    CuTe kernel (kernels/matmul.cu:71, alignment test kernels/gemm_cute.cu:302).
    That kernel made an illegal address access on a B200 (its 128-thread copy
    layouts under a 256-thread MMA, kernels/gemm_cute.cu:211-249), so those calls
    are refused before any launch; the per-row GEMV fallback stays usable."""
    return M > 1 and M % 128 == 0 and N % 128 == 0 and K % 32 == 0


class RefKernels:
    """The reference's own bf16 kernels (built from its sources; GPU only).

    Pointers are raw device addresses (ints)."""

    def __init__(self, cute: bool = False):
        self.cute = cute
        path = REF_CUTE if cute else REF_CUBLAS
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        self.lib = ctypes.CDLL(os.fspath(path), mode=os.RTLD_LOCAL | os.RTLD_NOW)
        L = self.lib
        L.ref_matmul.argtypes = [_vp, _vp, _vp, _i, _i, _i]
        L.ref_fused_silu_mul.argtypes = [_vp, _vp, _vp, _i, _i]
        L.ref_add.argtypes = [_vp, _vp, _i]
        L.ref_bf16_to_fp32.argtypes = [_vp, _vp, _i]
        L.ref_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float,
                                    _i, _i]
        L.ref_rmsnorm.argtypes = [_vp, _vp, _vp, _i, _i, ctypes.c_float]
        L.ref_rope.argtypes = [_vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float]
        L.ref_embedding.argtypes = [_vp, _vp, _vp, _i, _i]
        L.ref_argmax.argtypes = [_vp, _vp, _i]
        for n in ("ref_matmul", "ref_fused_silu_mul", "ref_add",
                  "ref_bf16_to_fp32", "ref_attention", "ref_rmsnorm", "ref_rope",
                  "ref_embedding", "ref_argmax", "ref_sync"):
            getattr(L, n).restype = _i

    def _ok(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what}: CUDA error {rc}")

    def matmul(self, C: int, A: int, B: int, M: int, N: int, K: int) -> None:
        if self.cute and cute_refused(M, N, K):
            raise ValueError(
                f"kernels::matmul {M}x{N}x{K} without cuBLAS would launch the reference's CuTe "
                "kernel (gemm_multi_stage), which accessed illegal addresses on a B200; refused")
        rc = self.lib.ref_matmul(C, A, B, M, N, K)
        if rc == REF_REFUSED_CUTE:
            raise ValueError(f"ref_matmul refused {M}x{N}x{K}: CuTe kernel shape")
        self._ok(rc, "kernels::matmul")

    def fused_silu_mul(self, out: int, g: int, u: int, seq: int, im: int) -> None:
        self._ok(self.lib.ref_fused_silu_mul(out, g, u, seq, im), "kernels::fused_silu_mul")

    def add(self, x: int, y: int, n: int) -> None:
        self._ok(self.lib.ref_add(x, y, n), "kernels::add")

    def bf16_to_fp32(self, out: int, inp: int, n: int) -> None:
        self._ok(self.lib.ref_bf16_to_fp32(out, inp, n), "kernels::bf16_to_fp32")

    def attention(self, out: int, q: int, k_pool: int, v_pool: int, seq_len: int,
                  cache_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                  scale: float, n_sink: int, window: int) -> None:
        self._ok(self.lib.ref_attention(out, q, k_pool, v_pool, seq_len, cache_len, num_heads,
                                        num_kv_heads, head_dim, scale, n_sink, window),
                 "kernels::attention")

    def rmsnorm(self, out: int, x: int, w: int, rows: int, dim: int, eps: float) -> None:
        self._ok(self.lib.ref_rmsnorm(out, x, w, rows, dim, eps), "kernels::rmsnorm")

    def rope(self, q: int, k: int, seq_len: int, num_heads: int, num_kv_heads: int,
             head_dim: int, start_pos: int, theta: float) -> None:
        self._ok(self.lib.ref_rope(q, k, seq_len, num_heads, num_kv_heads, head_dim, start_pos,
                                   theta), "kernels::rope")

    def embedding(self, out: int, table: int, ids: int, seq_len: int, hidden: int) -> None:
        self._ok(self.lib.ref_embedding(out, table, ids, seq_len, hidden), "kernels::embedding")

    def argmax(self, out: int, logits: int, n: int) -> None:
        self._ok(self.lib.ref_argmax(out, logits, n), "kernels::argmax")

    def sync(self) -> None:
        self._ok(self.lib.ref_sync(), "cudaDeviceSynchronize")
