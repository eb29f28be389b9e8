"""Safetensors files in the reference's format and names, and one layer in
the library's device layout (orininfer_b200/weights.py)."""
import json
import os
import struct

import numpy as np
import pytest
import torch

from orininfer_b200 import weights

SMALL = dict(hidden_size=64, intermediate_size=128, num_attention_heads=4,
             num_key_value_heads=2, head_dim=16, vocab_size=100)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_round_trip_and_reference_names(tmp_path, dtype):
    t, cfg = weights.synthetic_model(2, seed=3, dtype=dtype, **SMALL)
    weights.write_model_dir(str(tmp_path), t, cfg)
    back, meta = weights.read_safetensors(str(tmp_path / "model.safetensors"))
    assert meta == {"format": "pt"}
    assert list(back) == weights.reference_tensor_names(2)
    for name, x in t.items():
        y = back[name]
        assert y.dtype == x.dtype and y.shape == x.shape
        assert torch.equal(y.view(torch.uint8), x.contiguous().view(torch.uint8)), name
    c = json.load(open(tmp_path / "config.json"))
    for key in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads",
                "num_key_value_heads", "head_dim", "intermediate_size", "rms_norm_eps",
                "rope_theta", "tie_word_embeddings"):      # src/model_loader.cpp:216-226
        assert key in c, key
    assert c["num_hidden_layers"] == 2


def test_header_layout_matches_the_reference_parser(tmp_path):
    """8-byte little-endian header size, JSON header, data section right after
    it with every tensor's offsets relative to it and no holes
    (src/model_loader.cpp:238-302); the data starts 16-byte aligned."""
    t, cfg = weights.synthetic_model(1, seed=1, **SMALL)
    path = str(tmp_path / "m.safetensors")
    weights.write_safetensors(path, t)
    raw = open(path, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert (8 + n) % 16 == 0
    header = json.loads(raw[8:8 + n])
    spans = sorted(v["data_offsets"] for k, v in header.items() if k != "__metadata__")
    assert spans[0][0] == 0 and spans[-1][1] == len(raw) - 8 - n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    q = header["model.layers.0.self_attn.q_proj.weight"]
    assert q["dtype"] == "BF16" and q["shape"] == [64, 64]
    s, e = q["data_offsets"]
    got = np.frombuffer(raw[8 + n + s:8 + n + e], dtype=np.uint16)
    want = t["model.layers.0.self_attn.q_proj.weight"].view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, want.ravel())


def test_reader_rejects_a_hole(tmp_path):
    path = str(tmp_path / "hole.safetensors")
    js = json.dumps({"a": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)) + js + b"\0" * 8)
    with pytest.raises(ValueError):
        weights.read_safetensors(path)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2])
def test_layer_for_device_matches_separate_projections(world):
    """The device layout computes what the reference's seven projections do."""
    import orininfer_b200 as ob
    from oracle import oracle as orc
    from orininfer_b200 import tp
    from tests._util import EXACT_MIN, assert_close, bits, from_bits, seeded

    t, cfg = weights.synthetic_model(1, seed=7, dtype=torch.float16, **SMALL)
    x = seeded((8, 64), 9, 1.0)
    p = "model.layers.0"
    for rank in range(world):
        L = weights.layer_for_device(t, 0, cfg, "cuda:0", rank, world)
        qkv = ob.linear(x.cuda(), L["qkv"])
        wq, wk, wv = (t[f"{p}.self_attn.{n}_proj.weight"] for n in "qkv")
        ref = orc.linear(bits(x), bits(tp.shard_qkv(wq, wk, wv, 4, 2, 16, rank, world)), 0)
        assert_close(qkv.cpu().float(), from_bits(ref, torch.float16).float(), "qkv",
                     exact_min=EXACT_MIN)
        g, u = tp.shard_gate_up_rows(t[f"{p}.mlp.gate_proj.weight"],
                                     t[f"{p}.mlp.up_proj.weight"], rank, world)
        act = ob.linear(x.cuda(), L["gate_up"], epilogue="swiglu")
        ref = orc.linear(bits(x), orc.pack_gate_up(bits(g), bits(u)), 0, "swiglu")
        assert_close(act.cpu().float(), from_bits(ref, torch.float16).float(), "gate/up",
                     exact_min=EXACT_MIN)
        assert L["o_proj"].shape == (64, 64 // world) and L["down"].shape == (64, 128 // world)
