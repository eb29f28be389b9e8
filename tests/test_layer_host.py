"""Host-side checks of the layer drivers (orininfer_b200.layer), CPU only:
argument validation and the local shapes a tensor-parallel rank derives."""
import pytest
import torch

from orininfer_b200 import tp
from orininfer_b200.layer import DecoderLayer

CFG = dict(hidden_size=256, intermediate_size=256, num_attention_heads=4,
           num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-5, rope_theta=1e4)


def weights(cfg=CFG):
    H, IM = cfg["hidden_size"], cfg["intermediate_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    z = torch.zeros
    return {"qkv": z(qd + 2 * kvd, H, dtype=torch.float16), "o_proj": z(H, qd),
            "gate_up": z(2 * IM, H), "down": z(H, IM), "input_layernorm": z(H),
            "post_attention_layernorm": z(H)}


def test_max_tokens_bounded_by_the_ring():
    # the reference rejects calls longer than n_sink + window (src/kv_cache.cu:99-103)
    with pytest.raises(ValueError):
        DecoderLayer(weights(), CFG, n_sink=4, window=16, max_tokens=21)
    layer = DecoderLayer(weights(), CFG, n_sink=4, window=16, max_tokens=20)
    assert layer.k_pool.shape == (20, 2 * 64)
    assert layer.qkv.shape == (20, 4 * 64 + 2 * 2 * 64)


def test_qk_norm_needs_its_weights():
    with pytest.raises(ValueError):
        DecoderLayer(weights(), CFG, n_sink=4, window=16, max_tokens=8, qk_norm=True)
    w = weights()
    w["q_norm"] = torch.ones(64, dtype=torch.float16)
    w["k_norm"] = torch.ones(64, dtype=torch.float16)
    assert DecoderLayer(w, CFG, n_sink=4, window=16, max_tokens=8, qk_norm=True).qk_norm


@pytest.mark.parametrize("world,kv_local", [(1, 4), (2, 2), (4, 1), (8, 1)])
def test_tensor_parallel_local_heads_tinyllama(world, kv_local):
    """TinyLlama (32 query heads, 4 KV heads): every rank's query heads share
    the KV head(s) it holds, so its attention is local."""
    nh, nkv = 32, 4
    G = nh // nkv
    for rank in range(world):
        heads = range(rank * nh // world, (rank + 1) * nh // world)
        kv = tp.kv_heads_of(rank, world, nkv)
        assert len(kv) == kv_local
        assert sorted({h // G for h in heads}) == kv


def test_local_config_of_a_rank():
    from orininfer_b200.layer import TPDecoderLayer
    cfg = dict(hidden_size=2048, intermediate_size=5632, num_attention_heads=32,
               num_key_value_heads=4, head_dim=64)
    loc = TPDecoderLayer.local_config(cfg, 5, 8)
    assert (loc["num_attention_heads"], loc["num_key_value_heads"],
            loc["intermediate_size"], loc["hidden_size"]) == (4, 1, 704, 2048)
    with pytest.raises(ValueError):
        TPDecoderLayer.local_config(cfg, 0, 3)   # 32 heads don't split over 3 ranks


def test_prefill_chunks_follow_the_reference_engine():
    from orininfer_b200.layer import prefill_chunks
    # a 2048-token prompt with a 4 + 1024 cache: 1028 then 1020
    assert prefill_chunks(2048, 1028) == [(0, 1028), (1028, 1020)]
    assert prefill_chunks(5, 1028) == [(0, 5)]
    assert prefill_chunks(2056, 1028) == [(0, 1028), (1028, 1028)]
    assert prefill_chunks(0, 1028) == []
    with pytest.raises(ValueError):
        prefill_chunks(10, 0)


def test_rope_epilogue_taken_for_decode_calls_without_qk_norms():
    """Decode-sized calls of layers without q/k norms rotate and append q/k/v
    in the weight stream's epilogue (orin_linear_rope_append); calls with
    q/k norms (whole heads), longer calls, folded norms and head dims the
    epilogue is not built for keep the projection + orin_qkv_rope_append."""
    layer = DecoderLayer(weights(), CFG, n_sink=4, window=16, max_tokens=20)
    # a layer called back to back does not claim ORIN_ATTN_OWN_SLOTS_ONLY
    # (only Decoder, whose steps end with an ordinary launch, sets it)
    assert not layer.attn_own_slots
    assert layer._rope_in_epilogue(1, False)
    assert layer._rope_in_epilogue(DecoderLayer.ROPE_EPILOGUE_TOKENS, False)
    assert not layer._rope_in_epilogue(DecoderLayer.ROPE_EPILOGUE_TOKENS + 1, False)
    assert not layer._rope_in_epilogue(1, True)          # fold_norm path
    w = weights()
    w["q_norm"] = torch.ones(64, dtype=torch.float16)
    w["k_norm"] = torch.ones(64, dtype=torch.float16)
    qk = DecoderLayer(w, CFG, n_sink=4, window=16, max_tokens=8, qk_norm=True)
    assert not qk._rope_in_epilogue(1, False)
    cfg96 = dict(CFG, head_dim=96)
    odd = DecoderLayer(weights(cfg96), cfg96, n_sink=4, window=16, max_tokens=8)
    assert not odd._rope_in_epilogue(1, False)
