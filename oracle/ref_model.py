"""The reference's greedy generation loop run on the reference's own kernels.

TEST INFRASTRUCTURE ONLY: the token-for-token parity test uses this as the
checker for whole-model greedy decoding; nothing in orininfer_b200 imports it.

`RefModel` drives the kernels compiled from the reference's sources
(oracle/_ref/libref_cublas.so, its default cuBLAS build) through the call
sequence of the reference's engine, with the reference's buffers and rounding
points:

  Model::forward (src/model.cu:20-34): kernels::embedding, the layers,
  Model::lm_head_proj (src/model.cu:113-131): kernels::rmsnorm of all rows,
  kernels::matmul of the last row against lm_head (M = 1: gemv_kernel),
  kernels::bf16_to_fp32; the sampler's kernels::argmax (src/sampler.cu:24-27).

  Model::transformer_layer (src/model.cu:37-111): rmsnorm; q, k, v matmuls
  into the contiguous scratch (:56-61); rope (:70-73); the K/V append (:75);
  attention with scale 1/sqrtf(head_dim) (:79-84); o_proj matmul, add (:87-90);
  rmsnorm; gate and up matmuls, fused_silu_mul, down matmul, add (:95-110).
  The Qwen3 q/k RMSNorm (:64-67) runs only with qk_norm=True; TinyLlama has
  no q/k norm.

  Engine::run_generation (src/engine.cpp:55-115): the prompt in chunks of the
  cache's capacity n_sink + window (:71-81), the first token sampled from the
  last chunk's logits, then one forward of one token per step at position
  prompt_len + generated - 1 (:103).

The K/V append is KVCache::append_kv's scatter (src/kv_cache.cu:21-41): a
byte copy of row t into slot p (p < n_sink) or n_sink + (p - n_sink) % W of
position p = start_pos + t.  It is done here with a torch index copy, which
moves the same bytes; every other step runs the reference's kernel.
"""
from __future__ import annotations

import torch

from .oracle import RefKernels, ring_slot


class RefModel:
    """A TinyLlama/Qwen3-shaped model on the reference's kernels (bf16 only).

    tensors: the reference's tensor names (weights.reference_tensor_names),
    bf16, on any device; cfg: config.json keys.  Everything is copied to
    `device` once.  After forward(), `logits` holds the reference's fp32
    logits of the last row (16-bit rounded, then widened)."""

    def __init__(self, tensors, cfg, device, *, n_sink: int, window: int,
                 qk_norm: bool = False):
        self.k = RefKernels(cute=False)
        dev = torch.device(device)
        self.dev = dev
        self.cfg = dict(cfg)
        self.L = int(cfg["num_hidden_layers"])
        self.H = int(cfg["hidden_size"])
        self.IM = int(cfg["intermediate_size"])
        self.V = int(cfg["vocab_size"])
        self.nh = int(cfg["num_attention_heads"])
        self.nkv = int(cfg["num_key_value_heads"])
        self.hd = int(cfg.get("head_dim", self.H // self.nh))
        self.eps = float(cfg["rms_norm_eps"])
        self.theta = float(cfg["rope_theta"])
        self.n_sink, self.window = int(n_sink), int(window)
        self.capacity = self.n_sink + self.window
        self.qk_norm = bool(qk_norm)
        self.QD, self.KVD = self.nh * self.hd, self.nkv * self.hd

        def put(name):
            t = tensors[name]
            if t.dtype != torch.bfloat16:
                raise ValueError("the reference's kernels are bf16 only")
            return t.to(dev).contiguous()

        self.embed = put("model.embed_tokens.weight")
        self.final_norm = put("model.norm.weight")
        self.lm_head = put("lm_head.weight")
        self.layers = []
        for i in range(self.L):
            p = f"model.layers.{i}"
            lw = {n: put(f"{p}.{n}.weight") for n in (
                "input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                "self_attn.o_proj", "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj",
                "mlp.down_proj")}
            if self.qk_norm:
                lw["self_attn.q_norm"] = put(f"{p}.self_attn.q_norm.weight")
                lw["self_attn.k_norm"] = put(f"{p}.self_attn.k_norm.weight")
            lw["k_pool"] = torch.zeros((self.capacity, self.KVD), dtype=torch.bfloat16,
                                       device=dev)
            lw["v_pool"] = torch.zeros_like(lw["k_pool"])
            self.layers.append(lw)
        T = self.capacity
        bf = torch.bfloat16
        # ActivationPool's buffers (src/activation_pool.cu:19-48)
        self.x = torch.empty((T, self.H), dtype=bf, device=dev)          # buf_a
        self.buf_b = torch.empty((T * max(self.H, self.QD),), dtype=bf, device=dev)
        scratch = max(self.QD + 2 * self.KVD, 2 * self.IM, self.H) * T
        self.scratch = torch.empty((max(scratch, self.V),), dtype=bf, device=dev)
        self.logits = torch.empty((self.V,), dtype=torch.float32, device=dev)
        self.token = torch.empty((1,), dtype=torch.int32, device=dev)
        self.ids = torch.empty((T,), dtype=torch.int32, device=dev)
        # 1.0f / sqrtf((float)HD) as the reference computes it in fp32
        self.scale = float(torch.tensor(1.0, dtype=torch.float32)
                           / torch.sqrt(torch.tensor(float(self.hd), dtype=torch.float32)))

    def reset(self) -> None:
        """Empty KV pools (KVCache::reset)."""
        for lw in self.layers:
            lw["k_pool"].zero_()
            lw["v_pool"].zero_()

    # -- Model::transformer_layer ------------------------------------------------
    def _layer(self, i: int, S: int, start_pos: int) -> None:
        k, lw = self.k, self.layers[i]
        H, QD, KVD, IM, hd = self.H, self.QD, self.KVD, self.IM, self.hd
        x = self.x.data_ptr()
        bb = self.buf_b.data_ptr()
        sc = self.scratch
        q_buf = sc.data_ptr()
        k_off, v_off = S * QD, S * (QD + KVD)
        k_buf = sc[k_off:].data_ptr()
        v_buf = sc[v_off:].data_ptr()
        k.rmsnorm(bb, x, lw["input_layernorm"].data_ptr(), S, H, self.eps)
        k.matmul(q_buf, bb, lw["self_attn.q_proj"].data_ptr(), S, QD, H)
        k.matmul(k_buf, bb, lw["self_attn.k_proj"].data_ptr(), S, KVD, H)
        k.matmul(v_buf, bb, lw["self_attn.v_proj"].data_ptr(), S, KVD, H)
        if self.qk_norm:
            k.rmsnorm(q_buf, q_buf, lw["self_attn.q_norm"].data_ptr(), S * self.nh, hd, self.eps)
            k.rmsnorm(k_buf, k_buf, lw["self_attn.k_norm"].data_ptr(), S * self.nkv, hd,
                      self.eps)
        k.rope(q_buf, k_buf, S, self.nh, self.nkv, hd, start_pos, self.theta)
        # KVCache::append_kv: row t of the call into the slot of its position
        slots = torch.as_tensor(ring_slot(start_pos + torch.arange(S).numpy(), self.n_sink,
                                          self.window), device=self.dev)
        if torch.unique(slots).numel() != S:
            # two rows of one call share a slot (more than W window positions)
            raise ValueError("this call would overwrite its own slots")
        lw["k_pool"].index_copy_(0, slots, sc[k_off:k_off + S * KVD].view(S, KVD))
        lw["v_pool"].index_copy_(0, slots, sc[v_off:v_off + S * KVD].view(S, KVD))
        k.attention(bb, q_buf, lw["k_pool"].data_ptr(), lw["v_pool"].data_ptr(), S,
                    start_pos + S, self.nh, self.nkv, hd, self.scale, self.n_sink, self.window)
        k.matmul(q_buf, bb, lw["self_attn.o_proj"].data_ptr(), S, H, QD)
        k.add(x, q_buf, S * H)
        k.rmsnorm(bb, x, lw["post_attention_layernorm"].data_ptr(), S, H, self.eps)
        gate = q_buf
        up = sc[S * IM:].data_ptr()
        k.matmul(gate, bb, lw["mlp.gate_proj"].data_ptr(), S, IM, H)
        k.matmul(up, bb, lw["mlp.up_proj"].data_ptr(), S, IM, H)
        k.fused_silu_mul(gate, gate, up, S, IM)
        k.matmul(bb, gate, lw["mlp.down_proj"].data_ptr(), S, H, IM)
        k.add(x, bb, S * H)

    # -- Model::forward + the greedy sampler ---------------------------------------
    def forward(self, ids: torch.Tensor, start_pos: int) -> int:
        """One forward of len(ids) tokens at start_pos; returns the greedy token."""
        S = int(ids.numel())
        if S > self.capacity:
            raise ValueError("seq_len exceeds n_sink + window (src/kv_cache.cu:99-103)")
        self.ids[:S].copy_(ids.to(torch.int32))
        k = self.k
        k.embedding(self.x.data_ptr(), self.embed.data_ptr(), self.ids.data_ptr(), S, self.H)
        for i in range(self.L):
            self._layer(i, S, start_pos)
        bb = self.buf_b
        k.rmsnorm(bb.data_ptr(), self.x.data_ptr(), self.final_norm.data_ptr(), S, self.H,
                  self.eps)
        last = bb[(S - 1) * self.H:].data_ptr()
        k.matmul(self.scratch.data_ptr(), last, self.lm_head.data_ptr(), 1, self.V, self.H)
        k.bf16_to_fp32(self.logits.data_ptr(), self.scratch.data_ptr(), self.V)
        k.argmax(self.token.data_ptr(), self.logits.data_ptr(), self.V)
        k.sync()
        return int(self.token.item())

    def generate(self, prompt: list[int], max_new_tokens: int,
                 keep_logits: bool = False):
        """Engine::run_generation's greedy loop (no end token: TinyLlama-shaped
        random weights have none).  Returns the tokens, and with keep_logits
        also every step's fp32 logits stacked [steps, V] on the device."""
        self.reset()
        P = len(prompt)
        ids = torch.tensor(prompt, dtype=torch.int32)
        tok = 0
        for pos in range(0, P, self.capacity):
            n = min(self.capacity, P - pos)
            tok = self.forward(ids[pos:pos + n], pos)
        out = [tok]
        logits = [self.logits.clone()] if keep_logits else []
        one = torch.empty(1, dtype=torch.int32)
        while len(out) < max_new_tokens:
            one[0] = out[-1]
            out.append(self.forward(one, P + len(out) - 1))
            if keep_logits:
                logits.append(self.logits.clone())
        return (out, torch.stack(logits)) if keep_logits else out
