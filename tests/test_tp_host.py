"""Tensor-parallel sharding and reduction logic on the CPU (gloo, 2 ranks).

Each rank shards seeded weights exactly as bench.py / the engine would, runs
its shard in float64 (standing in for the kernel), and the partials of the
row-parallel projections are summed with a gloo all-reduce; the assembled
outputs must equal the unsharded layer."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from orininfer_b200 import tp
from orininfer_b200.synth import seeded

H, KVD, IM, NH, NKV, HD = 256, 64, 384, 8, 2, 32


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights():
    return dict(wq=seeded((H, H), 1, 0.02), wk=seeded((KVD, H), 2, 0.02),
                wv=seeded((KVD, H), 3, 0.02), wo=seeded((H, H), 4, 0.02),
                wg=seeded((IM, H), 5, 0.02), wu=seeded((IM, H), 6, 0.02),
                wd=seeded((H, IM), 7, 0.02))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _weights()
        x = seeded((5, H), 9, 1.0).double()
        attn = seeded((5, H), 10, 1.0).double()
        act = seeded((5, IM), 11, 1.0).double()
        # column-parallel q/k/v: this rank's heads
        qkv = x @ tp.shard_qkv(w["wq"], w["wk"], w["wv"], NH, NKV, HD, rank, world).double().T
        # row-parallel o/down: partial sums, then all-reduce
        qd = H // world
        po = attn[:, rank * qd:(rank + 1) * qd] @ tp.shard_cols(w["wo"], rank, world).double().T
        dist.all_reduce(po)
        imr = IM // world
        pd = act[:, rank * imr:(rank + 1) * imr] @ tp.shard_cols(w["wd"], rank, world).double().T
        dist.all_reduce(pd)
        g, u = tp.shard_gate_up_rows(w["wg"], w["wu"], rank, world)
        gu = x @ g.double().T, x @ u.double().T
        # numpy arrays travel by value (torch tensors would be shared through
        # file descriptors that vanish when this process exits)
        q.put((rank, qkv.numpy(), po.numpy(), pd.numpy(), (gu[0].numpy(), gu[1].numpy())))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_reassembles_the_layer():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict()
    for _ in range(world):
        r, qkv, po, pd, gu = q.get(timeout=120)
        res[r] = [torch.from_numpy(qkv), torch.from_numpy(po), torch.from_numpy(pd),
                  (torch.from_numpy(gu[0]), torch.from_numpy(gu[1]))]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = _weights()
    x = seeded((5, H), 9, 1.0).double()
    attn = seeded((5, H), 10, 1.0).double()
    act = seeded((5, IM), 11, 1.0).double()
    # row-parallel results identical on every rank and equal to the full GEMM
    for r in range(world):
        torch.testing.assert_close(res[r][1], attn @ w["wo"].double().T)
        torch.testing.assert_close(res[r][2], act @ w["wd"].double().T)
    # column-parallel q heads reassemble; KV heads split between the 2 ranks
    q_full = x @ w["wq"].double().T
    qd = H // world
    kv_per = KVD // world
    for r in range(world):
        got = res[r][0]
        torch.testing.assert_close(got[:, :qd], q_full[:, r * qd:(r + 1) * qd])
        k_full = x @ w["wk"].double().T
        torch.testing.assert_close(got[:, qd:qd + kv_per], k_full[:, r * kv_per:(r + 1) * kv_per])
    g_full = torch.cat([res[r][3][0] for r in range(world)], dim=1)
    torch.testing.assert_close(g_full, x @ w["wg"].double().T)


def test_kv_head_replication_when_ranks_exceed_kv_heads():
    assert tp.kv_heads_of(0, 8, 4) == [0] and tp.kv_heads_of(1, 8, 4) == [0]
    assert tp.kv_heads_of(7, 8, 4) == [3]
    assert tp.kv_heads_of(1, 2, 4) == [2, 3]
    with pytest.raises(ValueError):
        tp.kv_heads_of(0, 3, 4)


def test_shard_shapes_tinyllama_tp8():
    w = dict(wq=torch.zeros(2048, 2048, dtype=torch.float16), wk=torch.zeros(256, 2048, dtype=torch.float16),
             wv=torch.zeros(256, 2048, dtype=torch.float16))
    s = tp.shard_qkv(w["wq"], w["wk"], w["wv"], 32, 4, 64, 3, 8)
    assert s.shape == (256 + 64 + 64, 2048)
    g, u = tp.shard_gate_up_rows(torch.zeros(5632, 8), torch.zeros(5632, 8), 7, 8)
    assert g.shape == (704, 8)
    assert tp.shard_cols(torch.zeros(2048, 5632), 2, 8).shape == (2048, 704)


def test_ragged_vocab_split():
    parts = tp.ragged_split(128256, 8)
    assert parts[0] == (0, 16032) and parts[-1][1] == 128256
    parts = tp.ragged_split(32000, 3)
    assert sum(e - s for s, e in parts) == 32000 and max(e - s for s, e in parts) - min(e - s for s, e in parts) <= 1
    with pytest.raises(ValueError):
        tp.shard_rows(torch.zeros(10, 4), 0, 3)


def _layer_worker(rank, world, port, n_kv, q):
    """One rank of the tensor-parallel layer (orininfer_b200.layer.TPDecoderLayer's
    split), run with the oracle's pieces: this rank's heads and pools, fp32
    partials of o_proj and down summed over gloo, then the residual add and one
    rounding."""
    import numpy as np

    from oracle import oracle as O
    from orininfer_b200 import weights as Wt
    from tests._util import bits

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dt = 0
        dims = dict(hidden_size=256, intermediate_size=256, num_attention_heads=4,
                    num_key_value_heads=n_kv, head_dim=64, vocab_size=100)
        tensors, cfg = Wt.synthetic_model(1, seed=21, dtype=torch.float16, **dims)
        p = "model.layers.0"
        t = {k: tensors[f"{p}.{v}.weight"] for k, v in {
            "in": "input_layernorm", "post": "post_attention_layernorm",
            "q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
            "o": "self_attn.o_proj", "g": "mlp.gate_proj", "u": "mlp.up_proj",
            "d": "mlp.down_proj"}.items()}
        nh, hd, H = cfg["num_attention_heads"], cfg["head_dim"], cfg["hidden_size"]
        nh_l = nh // world
        nkv_l = len(tp.kv_heads_of(rank, world, n_kv))
        qkv_w = bits(tp.shard_qkv(t["q"], t["k"], t["v"], nh, n_kv, hd, rank, world))
        g_w, u_w = (bits(a) for a in tp.shard_gate_up_rows(t["g"], t["u"], rank, world))
        o_w, d_w = bits(tp.shard_cols(t["o"], rank, world)), bits(tp.shard_cols(t["d"], rank, world))
        ns, W = 2, 8
        kp = np.zeros((ns + W, nkv_l * hd), np.uint16)
        vp = np.zeros_like(kp)
        eps, theta = cfg["rms_norm_eps"], cfg["rope_theta"]

        def row_parallel(a, w, x):
            part = torch.from_numpy(O.linear(a, w, dt, "f32_partial"))
            dist.all_reduce(part)
            return O.add(x, O.round16(part.numpy(), dt), dt)

        rng = np.random.default_rng(3)
        outs, pos = [], 0
        for S in (10, 1, 1, 1):
            x = O.round16(rng.standard_normal((S, H)).astype(np.float32), dt)
            xn = O.rmsnorm(x, bits(t["in"]), dt, eps)
            qkv = O.linear(xn, qkv_w, dt)
            qd, kvd = nh_l * hd, nkv_l * hd
            qq = O.rope(qkv[:, :qd].reshape(S, nh_l, hd), pos, theta, dt)
            kk = O.rope(qkv[:, qd:qd + kvd].reshape(S, nkv_l, hd), pos, theta, dt)
            O.kv_append(kp, vp, kk.reshape(S, kvd), np.ascontiguousarray(qkv[:, qd + kvd:]), pos,
                        ns, W)
            att = O.attention(qq, kp.reshape(-1, nkv_l, hd), vp.reshape(-1, nkv_l, hd), S,
                              pos + S, nh_l, nkv_l, hd, float(np.float32(1) / np.sqrt(np.float32(hd))),
                              ns, W, dt)
            x = row_parallel(att.reshape(S, qd), o_w, x)
            xn = O.rmsnorm(x, bits(t["post"]), dt, eps)
            h = O.silu_mul(O.linear(xn, g_w, dt), O.linear(xn, u_w, dt), dt)
            x = row_parallel(h, d_w, x)
            outs.append(x)
            pos += S
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_kv", [2, 1])
def test_two_rank_layer_with_attention_matches_the_unsharded_layer(n_kv):
    """Heads, their KV heads (replicated when ranks outnumber them), local ring
    pools through prefill and a wrapping window, and the row-parallel finish:
    both ranks end with the unsharded layer's output."""
    import numpy as np

    from oracle import oracle as O
    from orininfer_b200 import weights as Wt
    from tests._util import assert_close, bits, from_bits

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layer_worker, args=(r, world, port, n_kv, q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    got = dict(q.get(timeout=240) for _ in range(world))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    dims = dict(hidden_size=256, intermediate_size=256, num_attention_heads=4,
                num_key_value_heads=n_kv, head_dim=64, vocab_size=100)
    tensors, cfg = Wt.synthetic_model(1, seed=21, dtype=torch.float16, **dims)
    p = "model.layers.0"
    L = {k: bits(tensors[f"{p}.{v}.weight"]) for k, v in {
        "input_layernorm": "input_layernorm", "post_attention_layernorm":
        "post_attention_layernorm", "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj",
        "v_proj": "self_attn.v_proj", "o_proj": "self_attn.o_proj", "gate_proj": "mlp.gate_proj",
        "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}.items()}
    ns, W = 2, 8
    kvd = n_kv * cfg["head_dim"]
    kp = np.zeros((ns + W, kvd), np.uint16)
    vp = np.zeros_like(kp)
    rng = np.random.default_rng(3)
    pos = 0
    for i, S in enumerate((10, 1, 1, 1)):
        x = O.round16(rng.standard_normal((S, cfg["hidden_size"])).astype(np.float32), 0)
        ref = O.transformer_layer(x, L, kp, vp, pos, dict(cfg, n_sink=ns, window=W), 0)
        for r in range(world):
            assert_close(from_bits(got[r][i], torch.float16).float(),
                         from_bits(ref, torch.float16).float(), f"rank {r} call {i}")
        assert np.array_equal(got[0][i], got[1][i])  # every rank holds the same result
        pos += S
