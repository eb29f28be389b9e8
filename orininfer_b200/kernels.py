"""Host-side mirror of the reference's GEMM-path operator interface.

The reference exposes raw-pointer functions in ``namespace kernels``
(include/kernels.h:51-108); this module offers the same names with the same
argument meaning over torch tensors (torch supplies device memory and
streams), each a direct call into liborin_b200.so:

    matmul(C, A, B, M, N, K)                   kernels::matmul
    fused_silu_mul(out, gate, up, seq, im)     kernels::fused_silu_mul
    add(x, y, n)                               kernels::add
    bf16_to_fp32(out, inp, n)                  kernels::bf16_to_fp32

plus the fused entry points that replace the reference's call pairs in
src/model.cu (``linear`` with an epilogue), the gate/up packer, and the
attention between the q/k/v and o projections:

    attention(out, q, k_pool, v_pool, ...)     kernels::attention
    kv_append(k_pool, v_pool, k, v, ...)       KVCache::append_kv (pools explicit)
    embedding(out, table, ids, seq, hidden)    kernels::embedding
    rmsnorm(out, x, w, seq, dim, eps)          kernels::rmsnorm
    rope(q, k, seq, heads, kv_heads, ...)      kernels::rope
    qkv_rope_append(q_out, qkv, pools, ...)    q/k norm + rope + append in one launch  fp16 and
bf16 are both accepted; the reference itself is bf16-only.

Errors raise ``OrinError`` (the library's status and message).  There is no
CPU path: tensors must live on a CUDA device.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import OrinError, check

_DTYPES = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
_EPILOGUES = {
    "none": _lib.EPI_NONE,
    "swiglu": _lib.EPI_SWIGLU,
    "residual": _lib.EPI_RESIDUAL,
    "f32": _lib.EPI_F32_OUT,
    "f32_partial": _lib.EPI_F32_PARTIAL,
}
_ALGOS = {
    "auto": _lib.ALGO_AUTO,
    "wide": _lib.ALGO_TC_WIDE,
    "skinny": _lib.ALGO_TC_SKINNY,
    "simt": _lib.ALGO_SIMT,
    "gemv": _lib.ALGO_GEMV,
}

__all__ = [
    "OrinError", "matmul", "fused_silu_mul", "add", "bf16_to_fp32", "linear", "linear_into",
    "pack_gate_up", "device_check", "plan_info", "lm_head_argmax", "attention",
    "attention_workspace_bytes", "kv_append", "rmsnorm", "rope", "qkv_rope_append",
    "embedding", "linear_rmsnorm", "attention_batch", "qkv_rope_append_batch",
    "linear_workspace", "linear_workspace_bytes",
]


def _ptr(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _stream(stream: Optional[torch.cuda.Stream]) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("orininfer_b200 kernels take CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise ValueError("orininfer_b200 kernels take contiguous tensors")


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; use float16 or bfloat16") from None


# ----------------------------------------------------------------- reference names

def matmul(C: torch.Tensor, A: torch.Tensor, B: torch.Tensor, M: int, N: int, K: int,
           stream: Optional[torch.cuda.Stream] = None) -> None:
    """C[M,N] = A[M,K] · B[N,K]^T (kernels/matmul.cu:47-81 semantics)."""
    _need_cuda(C, A, B)
    dt = _dtype_code(A)
    check(_lib.lib.orin_linear(_ptr(C), _ptr(A), _ptr(B), M, N, K, dt, _lib.EPI_NONE, None,
                               _stream(stream)))


def fused_silu_mul(out: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, seq_len: int,
                   intermediate_size: int, stream: Optional[torch.cuda.Stream] = None) -> None:
    """out = silu(gate) * up over seq_len*intermediate_size elements
    (kernels/fused_swiglu.cu:19-26); out may alias gate."""
    _need_cuda(out, gate, up)
    check(_lib.lib.orin_silu_mul(_ptr(out), _ptr(gate), _ptr(up), seq_len * intermediate_size,
                                 _dtype_code(gate), _stream(stream)))


def add(x: torch.Tensor, y: torch.Tensor, n: int,
        stream: Optional[torch.cuda.Stream] = None) -> None:
    """x += y elementwise, rounded (kernels/softmax.cu:78-83)."""
    _need_cuda(x, y)
    check(_lib.lib.orin_add(_ptr(x), _ptr(y), n, _dtype_code(x), _stream(stream)))


def bf16_to_fp32(out: torch.Tensor, inp: torch.Tensor, n: int,
                 stream: Optional[torch.cuda.Stream] = None) -> None:
    """out = float(inp) (kernels/softmax.cu:87-90); also accepts fp16 input."""
    _need_cuda(out, inp)
    check(_lib.lib.orin_widen_f32(_ptr(out), _ptr(inp), n, _dtype_code(inp), _stream(stream)))


# ----------------------------------------------------------------- fused entry points

def linear_workspace_bytes() -> int:
    """Workspace bytes that let linear_into(..., workspace=) pick any plan on the
    current GPU (orin_linear_workspace_bytes)."""
    n = ctypes.c_size_t(0)
    check(_lib.lib.orin_linear_workspace_bytes(ctypes.byref(n)))
    return int(n.value)


def linear_workspace(device=None) -> torch.Tensor:
    """A zeroed workspace for linear_into(..., workspace=) on `device`: its flag
    words must start at zero, and every call leaves them zero.  Calls sharing
    one workspace must be ordered on one stream."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    with torch.cuda.device(dev):
        n = linear_workspace_bytes()
    return torch.zeros(n, dtype=torch.uint8, device=dev)


def linear_into(out: torch.Tensor, x: torch.Tensor, w: torch.Tensor, *, epilogue: str = "none",
                residual: Optional[torch.Tensor] = None, algo: str = "auto",
                workspace: Optional[torch.Tensor] = None,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out = epilogue(x · w^T) written into `out` (see include/orin_b200.h).

    x [M, K]; w [N, K] ([2N, K] packed gate/up for "swiglu"); out [M, N]
    (float32 for "f32" / "f32_partial", else x.dtype); residual [M, N].
    With a workspace (linear_workspace()), prefill-sized problems may take the
    stream-K schedule (orin_linear_ws); algo must then be "auto".
    """
    _need_cuda(out, x, w, residual, workspace)
    dt = _dtype_code(x)
    if w.dtype != x.dtype or (residual is not None and residual.dtype != x.dtype):
        raise ValueError("x, w and residual must share one dtype")
    epi = _EPILOGUES[epilogue]
    M, K = x.shape
    N = out.shape[-1]
    if workspace is not None:
        if algo != "auto":
            raise ValueError("a workspace goes with algo='auto'")
        check(_lib.lib.orin_linear_ws(_ptr(out), _ptr(x), _ptr(w), M, N, K, dt, epi,
                                      _ptr(residual), _ptr(workspace),
                                      workspace.numel() * workspace.element_size(),
                                      _stream(stream)))
        return out
    check(_lib.lib.orin_linear_ex(_ptr(out), _ptr(x), _ptr(w), M, N, K, dt, epi, _ptr(residual),
                                  _ALGOS[algo], _stream(stream)))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, *, epilogue: str = "none",
           residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           algo: str = "auto", workspace: Optional[torch.Tensor] = None,
           stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Allocating form of linear_into."""
    M = x.shape[0]
    N = w.shape[0] // 2 if epilogue == "swiglu" else w.shape[0]
    if out is None:
        odt = torch.float32 if epilogue in ("f32", "f32_partial") else x.dtype
        out = torch.empty((M, N), dtype=odt, device=x.device)
    return linear_into(out, x, w, epilogue=epilogue, residual=residual, algo=algo,
                       workspace=workspace, stream=stream)


def linear_rmsnorm(out: torch.Tensor, x: torch.Tensor, w: torch.Tensor, norm: torch.Tensor,
                   eps: float, *, epilogue: str = "none",
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out = epilogue(rmsnorm(x; norm, eps) · w^T) with the norm folded into the
    decode weight stream (orin_linear_rmsnorm; M <= 32, epilogue "none" or
    "swiglu"): bit for bit rmsnorm() then linear_into()."""
    _need_cuda(out, x, w, norm)
    if len({x.dtype, w.dtype, norm.dtype}) != 1:
        raise ValueError("x, w and norm must share one dtype")
    M, K = x.shape
    check(_lib.lib.orin_linear_rmsnorm(_ptr(out), _ptr(x), _ptr(w), _ptr(norm), float(eps), M,
                                       out.shape[-1], K, _dtype_code(x), _EPILOGUES[epilogue],
                                       _stream(stream)))
    return out


def lm_head_argmax(h: torch.Tensor, w: torch.Tensor, *, keys: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None, norm: Optional[torch.Tensor] = None,
                   eps: float = 1e-5,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Greedy next token per row of h [M, K] through the LM head w [V, K]
    (orin_lm_head_argmax: the reference's LM head + bf16_to_fp32 + argmax,
    src/model.cu:113-131 and kernels/softmax.cu:52-73, with its tie-break).
    With `norm`, the final RMSNorm of h is folded in
    (orin_lm_head_argmax_rmsnorm)."""
    _need_cuda(h, w, keys, out, norm)
    if w.dtype != h.dtype:
        raise ValueError("h and w must share one dtype")
    M, K = h.shape
    V = w.shape[0]
    if keys is None:
        keys = torch.empty(M, dtype=torch.int64, device=h.device)
    if out is None:
        out = torch.empty(M, dtype=torch.int32, device=h.device)
    if norm is not None:
        check(_lib.lib.orin_lm_head_argmax_rmsnorm(_ptr(out), _ptr(h), _ptr(w), _ptr(norm),
                                                   float(eps), M, V, K, _dtype_code(h),
                                                   _ptr(keys), _stream(stream)))
        return out
    check(_lib.lib.orin_lm_head_argmax(_ptr(out), _ptr(h), _ptr(w), M, V, K, _dtype_code(h),
                                       _ptr(keys), _stream(stream)))
    return out


def embedding(out: torch.Tensor, table: torch.Tensor, token_ids: torch.Tensor, seq_len: int,
              hidden_size: int, stream: Optional[torch.cuda.Stream] = None) -> None:
    """kernels::embedding (include/kernels.h:12-19): out[t] = table[token_ids[t]]
    (int32 ids; an id outside the table gives a zero row)."""
    _need_cuda(out, table, token_ids)
    if token_ids.dtype != torch.int32:
        raise ValueError("token_ids must be int32")
    check(_lib.lib.orin_embedding(_ptr(out), _ptr(table), _ptr(token_ids), seq_len, hidden_size,
                                  table.shape[0], _stream(stream)))


def rmsnorm(out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, seq_len: int, dim: int,
            eps: float, stream: Optional[torch.cuda.Stream] = None) -> None:
    """kernels::rmsnorm (include/kernels.h:22-31): out = round16(x * r * w) per
    row, r = rsqrt(mean(x^2) + eps) (orin_rmsnorm)."""
    _need_cuda(out, x, weight)
    check(_lib.lib.orin_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), seq_len, dim, float(eps),
                                _dtype_code(x), _stream(stream)))


def rope(q: torch.Tensor, k: torch.Tensor, seq_len: int, num_heads: int, num_kv_heads: int,
         head_dim: int, start_pos: int, theta: float,
         stream: Optional[torch.cuda.Stream] = None) -> None:
    """kernels::rope (include/kernels.h:33-45): rotate-half rotary embedding
    in place on q [seq, heads, hd] and k [seq, kv_heads, hd] (orin_rope)."""
    _need_cuda(q, k)
    check(_lib.lib.orin_rope(_ptr(q), _ptr(k), seq_len, num_heads, num_kv_heads, head_dim,
                             start_pos, float(theta), _dtype_code(q), _stream(stream)))


def qkv_rope_append(q_out: torch.Tensor, qkv: torch.Tensor, k_pool: torch.Tensor,
                    v_pool: torch.Tensor, seq_len: int, start_pos: int, num_heads: int,
                    num_kv_heads: int, head_dim: int, theta: float, n_sink: int,
                    window_size: int, *, q_norm: Optional[torch.Tensor] = None,
                    k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
    """After the fused q/k/v projection (token rows [q | k | v]): optional
    per-head q/k RMSNorm, rotary embedding, q into q_out and k/v into their
    ring slots, in one launch (orin_qkv_rope_append)."""
    _need_cuda(q_out, qkv, k_pool, v_pool, q_norm, k_norm)
    check(_lib.lib.orin_qkv_rope_append(_ptr(q_out), _ptr(qkv), _ptr(q_norm), _ptr(k_norm),
                                        _ptr(k_pool), _ptr(v_pool), seq_len, start_pos,
                                        num_heads, num_kv_heads, head_dim, float(eps),
                                        float(theta), n_sink, window_size, _dtype_code(qkv),
                                        _stream(stream)))


def kv_append(k_pool: torch.Tensor, v_pool: torch.Tensor, k_src: torch.Tensor,
              v_src: torch.Tensor, seq_len: int, start_pos: int, n_sink: int,
              window_size: int, stream: Optional[torch.cuda.Stream] = None) -> None:
    """KVCache::append_kv with the pools passed explicitly (orin_kv_append):
    rows [seq_len, kv_dim] of positions start_pos.. into pool slots
    p (p < n_sink) or n_sink + (p - n_sink) % window_size
    (src/kv_cache.cu:21-41, 95-111)."""
    _need_cuda(k_pool, v_pool, k_src, v_src)
    if len({k_pool.dtype, v_pool.dtype, k_src.dtype, v_src.dtype}) != 1:
        raise ValueError("pools and sources must share one dtype")
    kv_dim = k_src.numel() // max(seq_len, 1)
    check(_lib.lib.orin_kv_append(_ptr(k_pool), _ptr(v_pool), _ptr(k_src), _ptr(v_src), seq_len,
                                  start_pos, n_sink, window_size, kv_dim, _dtype_code(k_src),
                                  _stream(stream)))


# orin_attention_batch_ex flag (include/orin_b200.h ORIN_ATTN_OWN_SLOTS_ONLY)
ATTN_OWN_SLOTS_ONLY = 1


def attention_workspace_bytes(seq_len: int, cache_len: int, num_heads: int, num_kv_heads: int,
                              head_dim: int, n_sink: int, window_size: int) -> int:
    """Device workspace that lets orin_attention split every few-token call."""
    n = ctypes.c_size_t(0)
    check(_lib.lib.orin_attention_workspace_bytes(ctypes.byref(n), seq_len, cache_len, num_heads,
                                                  num_kv_heads, head_dim, n_sink, window_size))
    return int(n.value)


def attention(out: torch.Tensor, q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
              seq_len: int, cache_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
              scale: float, n_sink: int, window_size: int, *,
              workspace: Optional[torch.Tensor] = None, split: bool = True,
              own_slots_only: bool = False,
              stream: Optional[torch.cuda.Stream] = None) -> None:
    """kernels::attention (include/kernels.h:58-80, kernels/attention.cu:27-175):
    sink + sliding-window GQA attention of q [seq_len, num_heads, head_dim]
    over the ring pools [n_sink + window_size, num_kv_heads, head_dim] into
    out.  With split (the default) few-token calls split their keys across
    CTAs through `workspace` (allocated here when not given; a caller's
    workspace must start zeroed: its first 4 KB are arrival counters that
    every call leaves zero).  own_slots_only: the kernel issued just before
    on the stream wrote only the slots of this call's own positions
    (ORIN_ATTN_OWN_SLOTS_ONLY: a single-token call loads the other keys
    before that kernel ends)."""
    _need_cuda(out, q, k_pool, v_pool, workspace)
    if len({out.dtype, q.dtype, k_pool.dtype, v_pool.dtype}) != 1:
        raise ValueError("out, q and the pools must share one dtype")
    ws_bytes = 0
    if split:
        if workspace is None:
            need = attention_workspace_bytes(seq_len, cache_len, num_heads, num_kv_heads,
                                             head_dim, n_sink, window_size)
            if need:
                workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        if workspace is not None:
            ws_bytes = workspace.numel() * workspace.element_size()
    else:
        workspace = None
    if own_slots_only:
        check(_lib.lib.orin_attention_batch_ex(
            _ptr(out), _ptr(q), _ptr(k_pool), _ptr(v_pool), 1, 0, seq_len, cache_len, num_heads,
            num_kv_heads, head_dim, float(scale), n_sink, window_size, _dtype_code(q),
            _ptr(workspace), ws_bytes, ATTN_OWN_SLOTS_ONLY, _stream(stream)))
        return
    check(_lib.lib.orin_attention(_ptr(out), _ptr(q), _ptr(k_pool), _ptr(v_pool), seq_len,
                                  cache_len, num_heads, num_kv_heads, head_dim, float(scale),
                                  n_sink, window_size, _dtype_code(q), _ptr(workspace), ws_bytes,
                                  _stream(stream)))


def attention_batch(out: torch.Tensor, q: torch.Tensor, k_pools: torch.Tensor,
                    v_pools: torch.Tensor, seq_len: int, cache_len: int, num_heads: int,
                    num_kv_heads: int, head_dim: int, scale: float, n_sink: int,
                    window_size: int, *, workspace: Optional[torch.Tensor] = None,
                    own_slots_only: bool = False,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
    """attention() over a batch of independent sequences in one launch
    (orin_attention_batch): q/out [batch, seq_len, num_heads, head_dim], pools
    [batch, n_sink + window_size, num_kv_heads, head_dim]; each sequence's
    result is bit-identical to its own attention() call.  own_slots_only as
    for attention()."""
    _need_cuda(out, q, k_pools, v_pools, workspace)
    if len({out.dtype, q.dtype, k_pools.dtype, v_pools.dtype}) != 1:
        raise ValueError("out, q and the pools must share one dtype")
    batch = k_pools.shape[0]
    if v_pools.shape != k_pools.shape or k_pools.stride(0) != v_pools.stride(0):
        raise ValueError("k_pools and v_pools must have one shape and stride")
    if workspace is None:
        need = batch * attention_workspace_bytes(seq_len, cache_len, num_heads, num_kv_heads,
                                                 head_dim, n_sink, window_size)
        if need:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(_lib.lib.orin_attention_batch_ex(_ptr(out), _ptr(q), _ptr(k_pools), _ptr(v_pools),
                                           batch, k_pools.stride(0), seq_len, cache_len,
                                           num_heads, num_kv_heads, head_dim, float(scale),
                                           n_sink, window_size, _dtype_code(q), _ptr(workspace),
                                           ws_bytes, ATTN_OWN_SLOTS_ONLY if own_slots_only else 0,
                                           _stream(stream)))


def qkv_rope_append_batch(q_out: torch.Tensor, qkv: torch.Tensor, k_pools: torch.Tensor,
                          v_pools: torch.Tensor, seq_len: int, start_pos: int, num_heads: int,
                          num_kv_heads: int, head_dim: int, theta: float, n_sink: int,
                          window_size: int, *, q_norm: Optional[torch.Tensor] = None,
                          k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6,
                          stream: Optional[torch.cuda.Stream] = None) -> None:
    """qkv_rope_append() for a batch of sequences at the same positions
    (orin_qkv_rope_append_batch): qkv/q_out rows [batch * seq_len], sequence
    b's K/V into k_pools[b] / v_pools[b]."""
    _need_cuda(q_out, qkv, k_pools, v_pools, q_norm, k_norm)
    if v_pools.shape != k_pools.shape or k_pools.stride(0) != v_pools.stride(0):
        raise ValueError("k_pools and v_pools must have one shape and stride")
    check(_lib.lib.orin_qkv_rope_append_batch(
        _ptr(q_out), _ptr(qkv), _ptr(q_norm), _ptr(k_norm), _ptr(k_pools), _ptr(v_pools),
        k_pools.shape[0], k_pools.stride(0), seq_len, start_pos, num_heads, num_kv_heads,
        head_dim, float(eps), float(theta), n_sink, window_size, _dtype_code(qkv),
        _stream(stream)))


def linear_rope_append(q_out: torch.Tensor, x: torch.Tensor, w_qkv: torch.Tensor,
                       k_pools: torch.Tensor, v_pools: torch.Tensor, seq_len: int,
                       start_pos: int, num_heads: int, num_kv_heads: int, head_dim: int,
                       theta: float, n_sink: int, window_size: int, *,
                       stream: Optional[torch.cuda.Stream] = None) -> None:
    """The q/k/v projection of x [batch * seq_len, hidden] with RoPE and the
    K/V append in the decode weight stream's epilogue
    (orin_linear_rope_append): the same results as linear_into(qkv, x, w_qkv)
    then qkv_rope_append_batch(q_out, qkv, k_pools, v_pools, ...) without q/k
    norms (src/model.cu:59-75).  k_pools / v_pools: [batch, n_sink + window,
    kv_dim] (or one pool [n_sink + window, kv_dim] for batch 1)."""
    _need_cuda(q_out, x, w_qkv, k_pools, v_pools)
    if v_pools.shape != k_pools.shape or k_pools.stride(0) != v_pools.stride(0):
        raise ValueError("k_pools and v_pools must have one shape and stride")
    batched = k_pools.dim() == 3
    batch = k_pools.shape[0] if batched else 1
    stride = k_pools.stride(0) if batched else 0
    if x.shape[0] != batch * seq_len:
        raise ValueError(f"x has {x.shape[0]} rows, expected batch * seq_len = "
                         f"{batch * seq_len}")
    check(_lib.lib.orin_linear_rope_append(
        _ptr(q_out), _ptr(x), _ptr(w_qkv), _ptr(k_pools), _ptr(v_pools), batch, stride, seq_len,
        start_pos, x.shape[1], num_heads, num_kv_heads, head_dim, float(theta), n_sink,
        window_size, _dtype_code(x), _stream(stream)))


def pack_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Interleave gate_proj and up_proj [IM, K] into the [2*IM, K] layout the
    fused SwiGLU epilogue reads (64-row gate/up groups)."""
    _need_cuda(w_gate, w_up)
    IM, K = w_gate.shape
    out = torch.empty((2 * IM, K), dtype=w_gate.dtype, device=w_gate.device)
    check(_lib.lib.orin_pack_gate_up(_ptr(out), _ptr(w_gate), _ptr(w_up), IM, K,
                                     _dtype_code(w_gate), _stream(stream)))
    return out


def plan_info(M: int, N: int, K: int, dtype: torch.dtype = torch.float16,
              epilogue: str = "none", algo: str = "auto", workspace_bytes: int = 0) -> dict:
    """The launch orin_linear (with a workspace of workspace_bytes:
    orin_linear_ws) would make for this problem on the current GPU."""
    info = (ctypes.c_int * 7)()
    check(_lib.lib.orin_plan_info_ws(M, N, K, _DTYPES[dtype], _EPILOGUES[epilogue], _ALGOS[algo],
                                     workspace_bytes, info))
    kind = {1: "tcgen05-wide", 2: "tcgen05-skinny", 3: "cuda-core", 4: "gemv"}[info[0]]
    return {"kernel": kind, "tile_cols": info[1], "cta_pair": bool(info[2]), "split_k": info[3],
            "grid": info[4], "tiles": info[5], "stream_k": bool(info[6])}


def device_check(stream: Optional[torch.cuda.Stream] = None) -> None:
    """Synchronise and raise if a kernel of this library gave up a bounded wait."""
    check(_lib.lib.orin_device_check(_stream(stream)))
