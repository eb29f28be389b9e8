"""The reference's transformer layer and model step on this library's kernels.

``DecoderLayer`` runs Model::transformer_layer (src/model.cu:37-111) for one
call of seq_len tokens at start_pos, on one GPU, in eight launches where the
reference makes fifteen:

    orin_rmsnorm(xn, x)                          :53
    orin_linear(qkv, xn, W_qkv)                  :59-61  (q/k/v weights stacked: one GEMM)
    orin_qkv_rope_append(q, qkv, pools)          :64-75  (Qwen3 q/k norm, RoPE, K/V append)
    orin_attention(att, q, pools)                :79-84  (decode splits merged in the kernel)
    orin_linear(x, att, W_o, RESIDUAL, x)        :87-90
    orin_rmsnorm(xn, x)                          :95
    orin_linear(h, xn, W_gate_up, SWIGLU)        :100-104
    orin_linear(x, h, W_down, RESIDUAL, x)       :107-110

with the reference's rounding points (the residual and SwiGLU epilogues round
where its separate add and fused_silu_mul kernels do).  Decode-sized calls
(up to 16 tokens) of layers without q/k norms put RoPE and the K/V append in
the q/k/v weight stream's epilogue (orin_linear_rope_append, the same values
bit for bit): seven launches.  With fold_norm, calls
of up to 16 tokens (decode) fold each RMSNorm into the projection after it
(orin_linear_rmsnorm: the decode weight stream normalises the rows it reads,
bit for bit the separate kernel's output), six launches; that is faster for
eagerly launched steps, but inside a CUDA graph the separate norm kernel
lets the projection stream its weights while the norm runs, so it is off by
default.  ``Decoder`` adds the embedding gather (:25), the final RMSNorm and
the LM head with the greedy argmax (:113-131 plus the sampler's argmax), i.e.
one Model::forward + greedy sample per call.  Every buffer is allocated once,
so a decode step can be captured in a CUDA graph.
"""
from __future__ import annotations

import math
from typing import Mapping, Optional

import torch

from . import kernels


def prefill_chunks(prompt_len: int, chunk: int) -> list[tuple[int, int]]:
    """(start position, length) of each prefill call: chunks of the KV cache's
    capacity n_sink + window, as Engine::generate splits a long prompt
    (src/engine.cpp:67-81)."""
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    return [(pos, min(chunk, prompt_len - pos)) for pos in range(0, prompt_len, chunk)]


class DecoderLayer:
    """One layer; `w` from weights.layer_for_device, `cfg` the model's
    config.json keys.  qk_norm applies q_norm / k_norm (Qwen3; the reference
    always does); Llama-family models (TinyLlama) have none.  With batch > 1
    the layer keeps one pair of ring pools per sequence (k_pools / v_pools
    [batch, n_sink + window, kv_dim]); forward(seq=b) runs sequence b alone
    (prefill), forward_batch one decode token of every sequence in one pass."""

    def __init__(self, w: Mapping[str, torch.Tensor], cfg: Mapping, *, n_sink: int, window: int,
                 max_tokens: int, qk_norm: bool = False,
                 workspace: Optional[torch.Tensor] = None, fold_norm: bool = False,
                 batch: int = 1, gemm_workspace: Optional[torch.Tensor] = None):
        self.w = dict(w)
        # stream-K workspace of the projections (kernels.linear_workspace),
        # shareable by every layer of a model run on one stream
        self.gemm_ws = gemm_workspace

        self.fold_norm = bool(fold_norm)
        self.nh = int(cfg["num_attention_heads"])
        self.nkv = int(cfg["num_key_value_heads"])
        self.hd = int(cfg.get("head_dim", cfg["hidden_size"] // self.nh))
        self.H = int(cfg["hidden_size"])
        self.IM = int(cfg["intermediate_size"])
        self.eps = float(cfg["rms_norm_eps"])
        self.theta = float(cfg["rope_theta"])
        self.n_sink, self.window = int(n_sink), int(window)
        if max_tokens > self.n_sink + self.window:
            raise ValueError("max_tokens exceeds n_sink + window (src/kv_cache.cu:99-103)")
        self.qk_norm = bool(qk_norm)
        # Set by a caller that orders consecutive calls fully (Decoder: every
        # step ends with an ordinary launch): a decode call's attention may
        # then load the pool slots other than the new token's before the
        # RoPE + append kernel ends (ORIN_ATTN_OWN_SLOTS_ONLY).  Off for calls
        # made back to back, where kernels launched early can still be
        # writing the previous call's slot.
        self.attn_own_slots = False
        if self.qk_norm and ("q_norm" not in self.w or "k_norm" not in self.w):
            raise ValueError("qk_norm needs q_norm and k_norm weights")
        qkv = self.w["qkv"]
        dev, dt = qkv.device, qkv.dtype
        QD, KVD = self.nh * self.hd, self.nkv * self.hd
        if batch < 1:
            raise ValueError("batch must be >= 1")
        self.batch = int(batch)
        self.k_pools = torch.zeros((self.batch, self.n_sink + self.window, KVD), dtype=dt,
                                   device=dev)
        self.v_pools = torch.zeros_like(self.k_pools)
        self.k_pool, self.v_pool = self.k_pools[0], self.v_pools[0]
        self.xn = torch.empty((max_tokens, self.H), dtype=dt, device=dev)
        self.qkv = torch.empty((max_tokens, QD + 2 * KVD), dtype=dt, device=dev)
        self.q = torch.empty((max_tokens, QD), dtype=dt, device=dev)
        self.att = torch.empty((max_tokens, QD), dtype=dt, device=dev)
        self.h = torch.empty((max_tokens, self.IM), dtype=dt, device=dev)
        self.scale = 1.0 / math.sqrt(self.hd)
        self.workspace = workspace

    @staticmethod
    def workspace_bytes(cfg: Mapping, n_sink: int, window: int, batch: int = 1) -> int:
        """Split-key workspace a decode step of `batch` sequences needs
        (shareable by all layers)."""
        nh = int(cfg["num_attention_heads"])
        hd = int(cfg.get("head_dim", cfg["hidden_size"] // nh))
        return batch * kernels.attention_workspace_bytes(1, n_sink + window + 64, nh,
                                                         int(cfg["num_key_value_heads"]), hd,
                                                         n_sink, window)

    # calls of at most this many tokens fold the norms into the weight stream
    FOLD_NORM_TOKENS = 16
    # calls of at most this many tokens rotate and append q/k/v in the weight
    # stream's epilogue (no q/k norms: those need whole heads)
    ROPE_EPILOGUE_TOKENS = 16

    def _rope_in_epilogue(self, tokens: int, fold: bool) -> bool:
        return (not fold and not self.qk_norm and tokens <= self.ROPE_EPILOGUE_TOKENS
                and self.hd in (64, 128) and self.H % 8 == 0)

    def forward(self, x: torch.Tensor, start_pos: int,
                stream: Optional[torch.cuda.Stream] = None, seq: int = 0) -> torch.Tensor:
        """x [seq_len, H] (the residual stream of sequence `seq`) is updated in
        place and returned."""
        S = x.shape[0]
        w = self.w
        xn, qkv, q, att = self.xn[:S], self.qkv[:S], self.q[:S], self.att[:S]
        k_pool, v_pool = self.k_pools[seq], self.v_pools[seq]
        fold = self.fold_norm and S <= self.FOLD_NORM_TOKENS
        if self._rope_in_epilogue(S, fold):
            kernels.rmsnorm(xn, x, w["input_layernorm"], S, self.H, self.eps, stream=stream)
            kernels.linear_rope_append(q, xn, w["qkv"], k_pool, v_pool, S, start_pos, self.nh,
                                       self.nkv, self.hd, self.theta, self.n_sink, self.window,
                                       stream=stream)
        else:
            if fold:
                kernels.linear_rmsnorm(qkv, x, w["qkv"], w["input_layernorm"], self.eps,
                                       stream=stream)
            else:
                kernels.rmsnorm(xn, x, w["input_layernorm"], S, self.H, self.eps, stream=stream)
                kernels.linear_into(qkv, xn, w["qkv"], workspace=self.gemm_ws, stream=stream)
            kernels.qkv_rope_append(q, qkv, k_pool, v_pool, S, start_pos, self.nh, self.nkv,
                                    self.hd, self.theta, self.n_sink, self.window,
                                    q_norm=w.get("q_norm") if self.qk_norm else None,
                                    k_norm=w.get("k_norm") if self.qk_norm else None,
                                    eps=self.eps, stream=stream)
        kernels.attention(att, q, k_pool, v_pool, S, start_pos + S, self.nh, self.nkv,
                          self.hd, self.scale, self.n_sink, self.window,
                          workspace=self.workspace, own_slots_only=self.attn_own_slots,
                          stream=stream)
        return self._mlp_tail(x, att, S, fold, stream)

    def forward_batch(self, x: torch.Tensor, start_pos: int,
                      stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """One decode token of each of the `batch` sequences, all at start_pos:
        x [batch, H] (row b = sequence b's residual stream) updated in place.
        The projections run once over all rows (the weights are streamed once
        per step, not once per sequence); RoPE + append and attention use each
        sequence's own pools.  Row b's result is bit-identical to
        forward(x[b:b+1], start_pos, seq=b)."""
        B = x.shape[0]
        if B != self.batch:
            raise ValueError(f"forward_batch takes {self.batch} rows, got {B}")
        w = self.w
        xn, qkv, q, att = self.xn[:B], self.qkv[:B], self.q[:B], self.att[:B]
        fold = self.fold_norm and B <= self.FOLD_NORM_TOKENS
        if self._rope_in_epilogue(B, fold):
            kernels.rmsnorm(xn, x, w["input_layernorm"], B, self.H, self.eps, stream=stream)
            kernels.linear_rope_append(q, xn, w["qkv"], self.k_pools, self.v_pools, 1, start_pos,
                                       self.nh, self.nkv, self.hd, self.theta, self.n_sink,
                                       self.window, stream=stream)
        else:
            if fold:
                kernels.linear_rmsnorm(qkv, x, w["qkv"], w["input_layernorm"], self.eps,
                                       stream=stream)
            else:
                kernels.rmsnorm(xn, x, w["input_layernorm"], B, self.H, self.eps, stream=stream)
                kernels.linear_into(qkv, xn, w["qkv"], stream=stream)
            kernels.qkv_rope_append_batch(q, qkv, self.k_pools, self.v_pools, 1, start_pos,
                                          self.nh, self.nkv, self.hd, self.theta, self.n_sink,
                                          self.window,
                                          q_norm=w.get("q_norm") if self.qk_norm else None,
                                          k_norm=w.get("k_norm") if self.qk_norm else None,
                                          eps=self.eps, stream=stream)
        kernels.attention_batch(att, q, self.k_pools, self.v_pools, 1, start_pos + 1, self.nh,
                                self.nkv, self.hd, self.scale, self.n_sink, self.window,
                                workspace=self.workspace,
                                own_slots_only=self.attn_own_slots, stream=stream)
        return self._mlp_tail(x, att, B, fold, stream)

    def _mlp_tail(self, x: torch.Tensor, att: torch.Tensor, S: int, fold: bool,
                  stream: Optional[torch.cuda.Stream]) -> torch.Tensor:
        """o_proj + residual, RMSNorm, gate/up + SwiGLU, down + residual."""
        w = self.w
        xn, h = self.xn[:S], self.h[:S]
        kernels.linear_into(x, att, w["o_proj"], epilogue="residual", residual=x,
                            workspace=self.gemm_ws, stream=stream)
        if fold:
            kernels.linear_rmsnorm(h, x, w["gate_up"], w["post_attention_layernorm"], self.eps,
                                   epilogue="swiglu", stream=stream)
        else:
            kernels.rmsnorm(xn, x, w["post_attention_layernorm"], S, self.H, self.eps,
                            stream=stream)
            kernels.linear_into(h, xn, w["gate_up"], epilogue="swiglu", workspace=self.gemm_ws,
                                stream=stream)
        kernels.linear_into(x, h, w["down"], epilogue="residual", residual=x,
                            workspace=self.gemm_ws, stream=stream)
        return x


class TPDecoderLayer(DecoderLayer):
    """DecoderLayer on one rank of a tensor-parallel group (one process per
    GPU), sharded as orininfer_b200.tp lays the projections out: this rank's
    query heads and their KV head(s) (replicated when ranks outnumber KV
    heads), with this rank's own ring pools; attention stays local; o_proj and
    down are row-parallel through `comm` (orin_tp_linear_row: fp32 partials
    summed over the ranks, then the residual add and one rounding, every rank
    receiving the whole [seq, H] result); gate/up is this rank's packed shard.
    `w` from weights.layer_for_device(..., rank, world)."""

    @staticmethod
    def local_config(cfg: Mapping, rank: int, world: int) -> dict:
        """The config this rank's shard looks like: its query heads, its KV
        head(s), its intermediate features (hidden size unchanged)."""
        from . import tp

        nh = int(cfg["num_attention_heads"])
        nkv = int(cfg["num_key_value_heads"])
        local = dict(cfg)
        local["num_attention_heads"] = tp.even_split(nh, world, "query heads")
        local["num_key_value_heads"] = len(tp.kv_heads_of(rank, world, nkv))
        local["intermediate_size"] = tp.even_split(int(cfg["intermediate_size"]), world,
                                                   "intermediate size")
        local["head_dim"] = int(cfg.get("head_dim", cfg["hidden_size"] // nh))
        return local

    def __init__(self, w: Mapping[str, torch.Tensor], cfg: Mapping, comm, *, n_sink: int,
                 window: int, max_tokens: int, qk_norm: bool = False,
                 workspace: Optional[torch.Tensor] = None):
        local = self.local_config(cfg, comm.rank, comm.world)
        super().__init__(w, local, n_sink=n_sink, window=window, max_tokens=max_tokens,
                         qk_norm=qk_norm, workspace=workspace)
        self.comm = comm
        self.partial = torch.empty((max_tokens, self.H), dtype=torch.float32,
                                   device=self.w["qkv"].device)

    def forward(self, x: torch.Tensor, start_pos: int,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """x [seq_len, H], the same on every rank, updated in place."""
        S = x.shape[0]
        w = self.w
        xn, qkv, q, att, h = self.xn[:S], self.qkv[:S], self.q[:S], self.att[:S], self.h[:S]
        partial = self.partial[:S]
        kernels.rmsnorm(xn, x, w["input_layernorm"], S, self.H, self.eps, stream=stream)
        kernels.linear_into(qkv, xn, w["qkv"], stream=stream)
        kernels.qkv_rope_append(q, qkv, self.k_pool, self.v_pool, S, start_pos, self.nh, self.nkv,
                                self.hd, self.theta, self.n_sink, self.window,
                                q_norm=w.get("q_norm") if self.qk_norm else None,
                                k_norm=w.get("k_norm") if self.qk_norm else None,
                                eps=self.eps, stream=stream)
        kernels.attention(att, q, self.k_pool, self.v_pool, S, start_pos + S, self.nh, self.nkv,
                          self.hd, self.scale, self.n_sink, self.window,
                          workspace=self.workspace, stream=stream)
        self.comm.linear_row(att, w["o_proj"], residual=x, out=x, partial=partial,
                             stream=stream)
        kernels.rmsnorm(xn, x, w["post_attention_layernorm"], S, self.H, self.eps, stream=stream)
        kernels.linear_into(h, xn, w["gate_up"], epilogue="swiglu", stream=stream)
        self.comm.linear_row(h, w["down"], residual=x, out=x, partial=partial, stream=stream)
        return x


class Decoder:
    """Model::forward + greedy sampling (src/model.cu:20-131): embedding,
    the layers, final RMSNorm and the LM head argmax of the last token."""

    def __init__(self, tensors: Mapping[str, torch.Tensor], cfg: Mapping, device, *,
                 n_sink: int, window: int, max_tokens: int, qk_norm: bool = False,
                 fold_norm: bool = False, batch: int = 1):
        from .weights import layer_for_device

        if max_tokens < batch:
            raise ValueError("max_tokens must cover one decode row per sequence")
        self.fold_norm = bool(fold_norm)
        self.batch = int(batch)
        self.cfg = dict(cfg)
        self.H = int(cfg["hidden_size"])
        self.eps = float(cfg["rms_norm_eps"])
        self.embed = tensors["model.embed_tokens.weight"].to(device)
        self.final_norm = tensors["model.norm.weight"].to(device)
        self.lm_head = tensors["lm_head.weight"].to(device)
        dt = self.embed.dtype
        ws = DecoderLayer.workspace_bytes(cfg, n_sink, window, self.batch)
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=device)
        self.gemm_ws = kernels.linear_workspace(device)
        self.layers = [
            DecoderLayer(layer_for_device(tensors, i, cfg, device), cfg, n_sink=n_sink,
                         window=window, max_tokens=max_tokens, qk_norm=qk_norm,
                         workspace=self.workspace, fold_norm=fold_norm, batch=self.batch,
                         gemm_workspace=self.gemm_ws)
            for i in range(int(cfg["num_hidden_layers"]))
        ]
        # every step ends with the argmax decode, an ordinary launch, so the
        # next step starts after the whole step has finished: within a step
        # only the new token's RoPE + append writes a layer's pools
        for layer in self.layers:
            layer.attn_own_slots = True
        self.x = torch.empty((max_tokens, self.H), dtype=dt, device=device)
        self.xn = torch.empty((self.batch, self.H), dtype=dt, device=device)
        self.keys = torch.empty(self.batch, dtype=torch.int64, device=device)
        self.tokens = torch.empty(self.batch, dtype=torch.int32, device=device)
        self.token = self.tokens[:1]

    def generate(self, prompt: list[int], max_new_tokens: int,
                 eos_ids: tuple[int, ...] = ()) -> list[int]:
        """Greedy generation as Engine::generate runs it (src/engine.cpp:55-115):
        the prompt prefilled in chunks of the cache's capacity, then one token
        per step until max_new_tokens or an end token.  Returns the generated
        ids; self.stats holds the prefill and decode times (ms)."""
        import time

        if not prompt or max_new_tokens < 1:
            return []
        dev = self.x.device
        ids = torch.tensor(prompt, dtype=torch.int32, device=dev)
        capacity = self.layers[0].n_sink + self.layers[0].window
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for pos, n in prefill_chunks(len(prompt), min(capacity, self.x.shape[0])):
            tok = self.step(ids[pos:pos + n], pos)
        out = [int(tok.item())]
        t1 = time.perf_counter()
        step_ids = torch.empty(1, dtype=torch.int32, device=dev)
        while len(out) < max_new_tokens and out[-1] not in eos_ids:
            step_ids.fill_(out[-1])
            tok = self.step(step_ids, len(prompt) + len(out) - 1)
            out.append(int(tok.item()))
        t2 = time.perf_counter()
        self.stats = {"prompt_tokens": len(prompt), "prefill_ms": (t1 - t0) * 1e3,
                      "generated_tokens": len(out), "decode_ms": (t2 - t1) * 1e3}
        return out

    def step(self, token_ids: torch.Tensor, start_pos: int,
             stream: Optional[torch.cuda.Stream] = None, seq: int = 0) -> torch.Tensor:
        """token_ids int32 [seq_len] of sequence `seq` on the device -> its next
        token id [1] (device)."""
        S = token_ids.shape[0]
        x = self.x[:S]
        kernels.embedding(x, self.embed, token_ids, S, self.H, stream=stream)
        for layer in self.layers:
            layer.forward(x, start_pos, stream=stream, seq=seq)
        return self._head(x[S - 1:S], self.xn[:1], self.keys[:1], self.tokens[seq:seq + 1],
                          stream)

    def step_batch(self, token_ids: torch.Tensor, start_pos: int,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """One decode step of every sequence: token_ids int32 [batch] (token b
        of sequence b, all at position start_pos) -> next tokens [batch]
        (device).  Each projection streams its weights once for the whole
        batch; token b equals what step(token_ids[b:b+1], start_pos, seq=b)
        gives."""
        B = token_ids.shape[0]
        if B != self.batch:
            raise ValueError(f"step_batch takes {self.batch} tokens, got {B}")
        x = self.x[:B]
        kernels.embedding(x, self.embed, token_ids, B, self.H, stream=stream)
        for layer in self.layers:
            layer.forward_batch(x, start_pos, stream=stream)
        return self._head(x, self.xn, self.keys, self.tokens, stream)

    def _head(self, rows: torch.Tensor, xn: torch.Tensor, keys: torch.Tensor,
              out: torch.Tensor, stream: Optional[torch.cuda.Stream]) -> torch.Tensor:
        """Final RMSNorm and the greedy LM head of `rows` into `out`."""
        n = rows.shape[0]
        if self.fold_norm:
            kernels.lm_head_argmax(rows, self.lm_head, keys=keys, out=out,
                                   norm=self.final_norm, eps=self.eps, stream=stream)
        else:
            kernels.rmsnorm(xn, rows, self.final_norm, n, self.H, self.eps, stream=stream)
            kernels.lm_head_argmax(xn, self.lm_head, keys=keys, out=out, stream=stream)
        return out

    def generate_batch(self, prompts: list[list[int]], max_new_tokens: int,
                       eos_ids: tuple[int, ...] = ()) -> list[list[int]]:
        """Greedy generation for `batch` prompts of one length: each prompt
        prefilled on its own (the chunks of generate()), then one batched
        decode step per token for all sequences together.  A sequence that
        emits an end token stops there (its row keeps being computed until
        every sequence has stopped, and what it computes is dropped).  Returns
        the generated ids per sequence; self.stats holds the times (ms)."""
        import time

        if len(prompts) != self.batch:
            raise ValueError(f"generate_batch takes {self.batch} prompts, got {len(prompts)}")
        lens = {len(p) for p in prompts}
        if len(lens) != 1 or 0 in lens:
            raise ValueError("the prompts of one batch must be non-empty and of one length")
        if max_new_tokens < 1:
            return [[] for _ in prompts]
        P = lens.pop()
        dev = self.x.device
        capacity = self.layers[0].n_sink + self.layers[0].window
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for b, prompt in enumerate(prompts):
            ids = torch.tensor(prompt, dtype=torch.int32, device=dev)
            for pos, n in prefill_chunks(P, min(capacity, self.x.shape[0])):
                self.step(ids[pos:pos + n], pos, seq=b)
        out = [[t] for t in self.tokens.tolist()]
        t1 = time.perf_counter()
        done = [o[-1] in eos_ids for o in out]
        step_ids = torch.empty(self.batch, dtype=torch.int32, device=dev)
        steps = 0
        while len(out[0]) < max_new_tokens and not all(done):
            step_ids.copy_(torch.tensor([o[-1] for o in out], dtype=torch.int32))
            tok = self.step_batch(step_ids, P + len(out[0]) - 1).tolist()
            steps += 1
            for b in range(self.batch):
                out[b].append(tok[b])
                done[b] = done[b] or tok[b] in eos_ids
        for b in range(self.batch):
            for i, t in enumerate(out[b]):
                if t in eos_ids:
                    del out[b][i + 1:]
                    break
        t2 = time.perf_counter()
        self.stats = {"prompt_tokens": P * self.batch, "prefill_ms": (t1 - t0) * 1e3,
                      "decode_steps": steps, "generated_tokens": sum(map(len, out)),
                      "decode_ms": (t2 - t1) * 1e3}
        return out


class TPDecoder(Decoder):
    """Decoder on one rank of a tensor-parallel group: the embedding and the
    final RMSNorm replicated, the layers as TPDecoderLayer, the LM head split by
    vocabulary rows (tp.ragged_split) with the greedy argmax combined over the
    ranks as one 64-bit key per token (TPComm.lm_head_argmax), so every rank
    gets the unsharded model's token."""

    def __init__(self, tensors: Mapping[str, torch.Tensor], cfg: Mapping, comm, device, *,
                 n_sink: int, window: int, max_tokens: int, qk_norm: bool = False):
        from . import tp
        from .weights import layer_for_device

        rank, world = comm.rank, comm.world
        self.comm = comm
        self.fold_norm = False
        self.cfg = dict(cfg)
        self.H = int(cfg["hidden_size"])
        self.eps = float(cfg["rms_norm_eps"])
        self.embed = tensors["model.embed_tokens.weight"].to(device)
        self.final_norm = tensors["model.norm.weight"].to(device)
        head = tensors["lm_head.weight"]
        lo, hi = tp.ragged_split(head.shape[0], world)[rank]
        self.v_offset = lo
        self.lm_head = head[lo:hi].contiguous().to(device)
        dt = self.embed.dtype
        local = TPDecoderLayer.local_config(cfg, rank, world)
        ws = DecoderLayer.workspace_bytes(local, n_sink, window)
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=device)
        self.layers = [
            TPDecoderLayer(layer_for_device(tensors, i, cfg, device, rank, world), cfg, comm,
                           n_sink=n_sink, window=window, max_tokens=max_tokens,
                           qk_norm=qk_norm, workspace=self.workspace)
            for i in range(int(cfg["num_hidden_layers"]))
        ]
        self.x = torch.empty((max_tokens, self.H), dtype=dt, device=device)
        self.xn = torch.empty((1, self.H), dtype=dt, device=device)
        self.keys = torch.empty(1, dtype=torch.int64, device=device)
        self.token = torch.empty(1, dtype=torch.int32, device=device)

    def step(self, token_ids: torch.Tensor, start_pos: int,
             stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """token_ids int32 [seq_len] (the same on every rank) -> next token [1]."""
        S = token_ids.shape[0]
        x = self.x[:S]
        kernels.embedding(x, self.embed, token_ids, S, self.H, stream=stream)
        for layer in self.layers:
            layer.forward(x, start_pos, stream=stream)
        kernels.rmsnorm(self.xn, x[S - 1:S], self.final_norm, 1, self.H, self.eps, stream=stream)
        self.comm.lm_head_argmax(self.xn, self.lm_head, self.v_offset, keys=self.keys,
                                 out=self.token, stream=stream)
        return self.token
