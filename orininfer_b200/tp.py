"""Tensor parallelism for the linear layers: weight sharding and the NCCL
communicator of liborin_b200.so.

Layout (one process per GPU, rank r of W):
  * q/k/v  — column-parallel by attention head.  Each rank keeps n_heads/W
    query heads and n_kv/W key/value heads; when W > n_kv (TinyLlama's 4 KV
    heads on 8 GPUs) each KV head is replicated on W/n_kv consecutive ranks.
  * gate/up — column-parallel by intermediate feature (IM/W per rank), packed
    per shard so the fused SwiGLU stays local to the rank.
  * o/down — row-parallel (split along K).  Each rank produces an fp32 partial
    [M, H]; the partials are summed over the ranks (over NVLink peer memory
    after TPComm.enable_p2p, else ncclAllReduce), then the residual add and
    the single rounding to 16 bits follow (orin_tp_linear_row).
  * LM head — column-parallel by vocabulary row (any split, ragged tail ok);
    greedy decoding reduces each rank's best token to one 64-bit key and
    combines the ranks' keys with one max all-reduce (TPComm.lm_head_argmax).

The reference is single-GPU (include/kv_cache.h:7); this module has no
counterpart there.  Sharding helpers are plain torch and run on any device.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import check
from .kernels import _dtype_code, _need_cuda, _ptr, _stream, pack_gate_up


def even_split(total: int, world: int, what: str = "dimension") -> int:
    if total % world != 0:
        raise ValueError(f"{what} {total} does not split evenly over {world} ranks")
    return total // world


def ragged_split(total: int, world: int) -> list[tuple[int, int]]:
    """[start, stop) per rank, sizes differing by at most one (vocab rows)."""
    base, rem = divmod(total, world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((s, s + n))
        s += n
    return out


def kv_heads_of(rank: int, world: int, n_kv: int) -> list[int]:
    """KV heads rank `rank` holds: a block of n_kv/W heads, or one replicated
    head when W > n_kv."""
    if world <= n_kv:
        per = even_split(n_kv, world, "KV heads")
        return list(range(rank * per, (rank + 1) * per))
    if world % n_kv != 0:
        raise ValueError(f"{world} ranks can't replicate {n_kv} KV heads evenly")
    return [rank // (world // n_kv)]


def shard_qkv(wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, n_heads: int, n_kv: int,
              head_dim: int, rank: int, world: int) -> torch.Tensor:
    """Fused [q_shard; k_shard; v_shard] rows for rank `rank`."""
    qh = even_split(n_heads, world, "query heads")
    q = wq[rank * qh * head_dim:(rank + 1) * qh * head_dim]
    kv = kv_heads_of(rank, world, n_kv)
    k = torch.cat([wk[h * head_dim:(h + 1) * head_dim] for h in kv])
    v = torch.cat([wv[h * head_dim:(h + 1) * head_dim] for h in kv])
    return torch.cat([q, k, v]).contiguous()


def shard_rows(w: torch.Tensor, rank: int, world: int, ragged: bool = False) -> torch.Tensor:
    """Column-parallel shard: a block of output rows of w [N, K]."""
    if ragged:
        s, e = ragged_split(w.shape[0], world)[rank]
        return w[s:e].contiguous()
    n = even_split(w.shape[0], world, "output rows")
    return w[rank * n:(rank + 1) * n].contiguous()


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row-parallel shard: a block of input columns of w [N, K]."""
    k = even_split(w.shape[1], world, "input columns")
    return w[:, rank * k:(rank + 1) * k].contiguous()


def shard_gate_up_rows(w_gate: torch.Tensor, w_up: torch.Tensor, rank: int,
                       world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """This rank's gate/up rows (before packing)."""
    im = even_split(w_gate.shape[0], world, "intermediate size")
    if im % 64 != 0:
        raise ValueError(f"per-rank intermediate size {im} is not a multiple of 64")
    sl = slice(rank * im, (rank + 1) * im)
    return w_gate[sl].contiguous(), w_up[sl].contiguous()


def shard_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, rank: int,
                  world: int) -> torch.Tensor:
    """This rank's packed gate/up weight for the fused SwiGLU (CUDA tensors)."""
    g, u = shard_gate_up_rows(w_gate, w_up, rank, world)
    return pack_gate_up(g, u)


def exchange_unique_id(rank: int, group=None) -> bytes:
    """Rank 0 creates an NCCL unique id and broadcasts it over an initialised
    torch.distributed process group (any backend)."""
    import torch.distributed as dist

    obj: list = [TPComm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


class TPComm:
    """This rank's NCCL communicator (orin_tp_* in include/orin_b200.h)."""

    def __init__(self, rank: int, world: int, device: int, unique_id: bytes,
                 timeout_s: float = 60.0):
        if len(unique_id) != _lib.TP_UNIQUE_ID_BYTES:
            raise ValueError("unique_id must be the 128 bytes orin_tp_unique_id returned")
        self.rank, self.world, self.device = rank, world, device
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, _lib.TP_UNIQUE_ID_BYTES)
        check(_lib.lib.orin_tp_init(ctypes.byref(h), buf, rank, world, device, float(timeout_s)))
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(_lib.TP_UNIQUE_ID_BYTES)
        check(_lib.lib.orin_tp_unique_id(buf))
        return buf.raw

    def allreduce_f32(self, t: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> None:
        _need_cuda(t)
        if t.dtype != torch.float32:
            raise ValueError("allreduce_f32 takes float32 tensors")
        check(_lib.lib.orin_tp_allreduce_f32(self._h, _ptr(t), t.numel(), _stream(stream)))

    def linear_row(self, x_shard: torch.Tensor, w_shard: torch.Tensor, *,
                   residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                   partial: Optional[torch.Tensor] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Row-parallel linear: out = round16(residual + round16(sum_r x_r · w_r^T))."""
        _need_cuda(x_shard, w_shard, residual, out, partial)
        M, Ks = x_shard.shape
        N = w_shard.shape[0]
        if out is None:
            out = torch.empty((M, N), dtype=x_shard.dtype, device=x_shard.device)
        if partial is None:
            partial = torch.empty((M, N), dtype=torch.float32, device=x_shard.device)
        check(_lib.lib.orin_tp_linear_row(self._h, _ptr(out), _ptr(x_shard), _ptr(w_shard), M, N,
                                          Ks, _dtype_code(x_shard), _ptr(residual),
                                          _ptr(partial), _stream(stream)))
        return out

    def lm_head_argmax(self, h: torch.Tensor, w_shard: torch.Tensor, v_offset: int, *,
                       keys: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                       stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Greedy token per row of h with the LM head split by vocabulary rows:
        this rank holds rows [v_offset, v_offset + len(w_shard)) (orin_tp_lm_head_argmax)."""
        _need_cuda(h, w_shard, keys, out)
        M, K = h.shape
        if keys is None:
            keys = torch.empty(M, dtype=torch.int64, device=h.device)
        if out is None:
            out = torch.empty(M, dtype=torch.int32, device=h.device)
        check(_lib.lib.orin_tp_lm_head_argmax(self._h, _ptr(out), _ptr(h), _ptr(w_shard), M,
                                              w_shard.shape[0], int(v_offset), K,
                                              _dtype_code(h), _ptr(keys), _stream(stream)))
        return out

    def enable_p2p(self, max_elems: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Collective: reduce row-parallel calls of up to max_elems outputs over
        NVLink peer memory instead of NCCL (orin_tp_enable_p2p)."""
        check(_lib.lib.orin_tp_enable_p2p(self._h, int(max_elems), _stream(stream)))

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        check(_lib.lib.orin_tp_wait(self._h, _stream(stream)))

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, None
            check(_lib.lib.orin_tp_destroy(h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
