"""Model weights on disk: safetensors files the reference loads, and the
library's layout on the device.

The reference maps ``model.safetensors`` (src/model_loader.cpp:238-302): an
8-byte little-endian header length, a JSON header
``{name: {"dtype", "shape", "data_offsets": [start, end]}}`` (offsets relative
to the data section that follows the header), then the raw tensor bytes; it
skips ``__metadata__``.  Its WeightStore (src/weight_store.cu:59-80) reads the
tensors named below as bf16, and ModelLoader::parse_config
(src/model_loader.cpp:198-231) the config keys below.

* ``write_safetensors`` / ``read_safetensors``: the file format (no holes in
  the data section; the header is padded with spaces so the data starts on a
  16-byte boundary, which keeps every tensor whose size is a multiple of 16
  bytes 16-byte aligned).
* ``reference_tensor_names`` / ``synthetic_model``: the tensor set of an
  ``n_layers`` model with seeded random-init weights (projections and
  embeddings ~N(0, 0.02), norm weights 1), plus a ``config.json`` for it.
  TinyLlama has no q/k norms; the reference's loader requires them, so they
  are written as ones.
* ``layer_for_device``: one layer in this library's layout (q/k/v rows
  concatenated, gate/up packed for the fused SwiGLU epilogue), optionally as
  this rank's tensor-parallel shard.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Mapping, Optional

import numpy as np
import torch

_ST_DTYPES = {torch.float16: "F16", torch.bfloat16: "BF16", torch.float32: "F32"}
_ST_FROM = {v: k for k, v in _ST_DTYPES.items()}

TINYLLAMA = dict(hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
                 num_attention_heads=32, num_key_value_heads=4, head_dim=64,
                 vocab_size=32000, rms_norm_eps=1e-5, rope_theta=10000.0,
                 max_position_embeddings=2048, tie_word_embeddings=False)


def write_safetensors(path: str, tensors: Mapping[str, torch.Tensor],
                      metadata: Optional[Mapping[str, str]] = None) -> None:
    """Write tensors (CPU or CUDA, float16 / bfloat16 / float32) in order."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs = []
    off = 0
    for name, t in tensors.items():
        if t.dtype not in _ST_DTYPES:
            raise ValueError(f"{name}: unsupported dtype {t.dtype}")
        b = t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()
        header[name] = {"dtype": _ST_DTYPES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    js = json.dumps(header, separators=(",", ":")).encode()
    js += b" " * ((-(8 + len(js))) % 16)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """Tensors (CPU, sharing one read of the file) and the metadata."""
    with open(path, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n].decode())
    data = memoryview(raw)[8 + n:]
    meta = header.pop("__metadata__", {}) or {}
    out = {}
    end_max = 0
    for name, info in header.items():
        dt = _ST_FROM.get(info["dtype"])
        if dt is None:
            raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
        start, end = info["data_offsets"]
        arr = np.frombuffer(data[start:end], dtype=np.uint8).copy()
        out[name] = torch.from_numpy(arr).view(dt).reshape(info["shape"])
        end_max = max(end_max, end)
    if end_max != len(data):
        raise ValueError("data section has bytes no tensor covers")
    return out, meta


def reference_tensor_names(n_layers: int) -> list[str]:
    """Every tensor the reference's WeightStore loads (src/weight_store.cu:60-80)."""
    names = ["model.embed_tokens.weight"]
    for i in range(n_layers):
        p = f"model.layers.{i}"
        names += [f"{p}.input_layernorm.weight", f"{p}.self_attn.q_proj.weight",
                  f"{p}.self_attn.q_norm.weight", f"{p}.self_attn.k_proj.weight",
                  f"{p}.self_attn.k_norm.weight", f"{p}.self_attn.v_proj.weight",
                  f"{p}.self_attn.o_proj.weight", f"{p}.post_attention_layernorm.weight",
                  f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight",
                  f"{p}.mlp.down_proj.weight"]
    return names + ["model.norm.weight", "lm_head.weight"]


def synthetic_model(n_layers: int, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
                    **dims) -> tuple[dict[str, torch.Tensor], dict]:
    """Seeded random-init weights of a TinyLlama-shaped model (dims override
    TINYLLAMA) in the reference's names, and its config.json contents."""
    cfg = dict(TINYLLAMA, **dims)
    cfg["num_hidden_layers"] = n_layers
    H, IM, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    hd = cfg["head_dim"]
    QD, KVD = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(shape, generator=g) * 0.02).to(dtype)

    def ones(n):
        return torch.ones(n, dtype=dtype)

    t = {"model.embed_tokens.weight": rnd(V, H)}
    for i in range(n_layers):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = ones(H)
        t[f"{p}.self_attn.q_proj.weight"] = rnd(QD, H)
        t[f"{p}.self_attn.q_norm.weight"] = ones(hd)
        t[f"{p}.self_attn.k_proj.weight"] = rnd(KVD, H)
        t[f"{p}.self_attn.k_norm.weight"] = ones(hd)
        t[f"{p}.self_attn.v_proj.weight"] = rnd(KVD, H)
        t[f"{p}.self_attn.o_proj.weight"] = rnd(H, QD)
        t[f"{p}.post_attention_layernorm.weight"] = ones(H)
        t[f"{p}.mlp.gate_proj.weight"] = rnd(IM, H)
        t[f"{p}.mlp.up_proj.weight"] = rnd(IM, H)
        t[f"{p}.mlp.down_proj.weight"] = rnd(H, IM)
    t["model.norm.weight"] = ones(H)
    t["lm_head.weight"] = rnd(V, H)
    return t, cfg


def write_model_dir(path: str, tensors: Mapping[str, torch.Tensor], cfg: Mapping) -> None:
    """model.safetensors + config.json in `path` (the reference also wants a
    tokenizer.json there, which is not on the linear-layer path)."""
    os.makedirs(path, exist_ok=True)
    write_safetensors(os.path.join(path, "model.safetensors"), tensors,
                      metadata={"format": "pt"})
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(dict(cfg), f, indent=2)


def layer_for_device(tensors: Mapping[str, torch.Tensor], layer: int, cfg: Mapping,
                     device, rank: int = 0, world: int = 1) -> dict[str, torch.Tensor]:
    """Layer `layer` in this library's layout on `device` (a CUDA device):
    "qkv" [q|k|v rows, H] (the reference's contiguous q/k/v scratch order,
    src/model.cu:56-58), "o_proj", "gate_up" (packed for the SwiGLU epilogue),
    "down"; with world > 1, this rank's tensor-parallel shard of each.  The
    norm weights ride along unsharded: "input_layernorm",
    "post_attention_layernorm" and, where the file has them, "q_norm" /
    "k_norm"."""
    from . import kernels, tp

    p = f"model.layers.{layer}"
    wq = tensors[f"{p}.self_attn.q_proj.weight"]
    wk = tensors[f"{p}.self_attn.k_proj.weight"]
    wv = tensors[f"{p}.self_attn.v_proj.weight"]
    wo = tensors[f"{p}.self_attn.o_proj.weight"]
    wg = tensors[f"{p}.mlp.gate_proj.weight"]
    wu = tensors[f"{p}.mlp.up_proj.weight"]
    wd = tensors[f"{p}.mlp.down_proj.weight"]
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    qkv = tp.shard_qkv(wq, wk, wv, nh, nkv, hd, rank, world)
    g, u = tp.shard_gate_up_rows(wg, wu, rank, world)
    out = {"qkv": qkv.to(device),
           "gate_up": kernels.pack_gate_up(g.to(device), u.to(device))}
    if world == 1:
        out["o_proj"] = wo.to(device)
        out["down"] = wd.to(device)
    else:
        out["o_proj"] = tp.shard_cols(wo, rank, world).to(device)
        out["down"] = tp.shard_cols(wd, rank, world).to(device)
    for name in ("input_layernorm", "post_attention_layernorm"):
        out[name] = tensors[f"{p}.{name}.weight"].to(device)
    for name in ("q_norm", "k_norm"):
        t = tensors.get(f"{p}.self_attn.{name}.weight")
        if t is not None:
            out[name] = t.to(device)
    return out
