"""The tensor-parallel layer (orininfer_b200.layer.TPDecoderLayer) on 2, 4 and 8
GPUs, one process per GPU: a TinyLlama layer split by heads (its 4 KV heads
replicated on pairs of ranks at 8), local ring pools, row-parallel o_proj and
down reduced over NVLink peer memory.  A 64-token prefill and three decode
tokens on every rank must give the unsharded oracle layer's output, and the
same bits on every rank.  Then the model step (TPDecoder, two layers, the LM
head split by vocabulary rows): every rank picks the same greedy token, one
whose oracle logit is within the tolerance of the oracle's best."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import numpy as np
    import torch.distributed as dist

    import orininfer_b200 as ob
    from oracle import oracle as O
    from orininfer_b200 import tp
    from orininfer_b200 import weights as Wt
    from orininfer_b200.layer import TPDecoderLayer
    from tests._util import assert_close, bits, from_bits

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        comm = tp.TPComm(rank, world, rank, tp.exchange_unique_id(rank), timeout_s=60.0)
        tensors, cfg = Wt.synthetic_model(1, seed=7, dtype=torch.float16)
        ns, W = 4, 64
        comm.enable_p2p((ns + W) * cfg["hidden_size"])
        layer = TPDecoderLayer(Wt.layer_for_device(tensors, 0, cfg, dev, rank, world), cfg, comm,
                               n_sink=ns, window=W, max_tokens=ns + W)
        p = "model.layers.0"
        L = {k: bits(tensors[f"{p}.{v}.weight"]) for k, v in {
            "input_layernorm": "input_layernorm",
            "post_attention_layernorm": "post_attention_layernorm",
            "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj",
            "v_proj": "self_attn.v_proj", "o_proj": "self_attn.o_proj",
            "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
            "down_proj": "mlp.down_proj"}.items()}
        kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
        kp = np.zeros((ns + W, kvd), np.uint16)
        vp = np.zeros_like(kp)
        rng = np.random.default_rng(11)
        pos = 0
        for S in (64, 1, 1, 1):
            x = O.round16(rng.standard_normal((S, cfg["hidden_size"])).astype(np.float32), 0)
            y = layer.forward(from_bits(x, torch.float16).to(dev), pos)
            comm.wait()
            ob.device_check()
            ref = O.transformer_layer(x, L, kp, vp, pos, dict(cfg, n_sink=ns, window=W), 0)
            assert_close(y.cpu().float(), from_bits(ref, torch.float16).float(),
                         f"rank {rank} at {pos} (+{S})")
            # every rank must hold the same bits: compare a checksum over gloo
            sig = torch.tensor([float(bits(y.cpu()).astype(np.int64).sum())], dtype=torch.float64)
            all_sig = [torch.zeros_like(sig) for _ in range(world)]
            dist.all_gather(all_sig, sig)
            assert all(float(a) == float(sig) for a in all_sig), "ranks disagree"
            pos += S
        torch.cuda.synchronize()
        del layer

        # the model step: two layers, vocabulary-parallel LM head with the greedy
        # argmax combined over the ranks
        from orininfer_b200.layer import TPDecoder
        dims = dict(vocab_size=3000)
        tensors, cfg = Wt.synthetic_model(2, seed=9, dtype=torch.float16, **dims)
        model = TPDecoder(tensors, cfg, comm, dev, n_sink=ns, window=W, max_tokens=ns + W)
        Ls = []
        for i in range(2):
            pi = f"model.layers.{i}"
            Ls.append({k: bits(tensors[f"{pi}.{v}.weight"]) for k, v in {
                "input_layernorm": "input_layernorm",
                "post_attention_layernorm": "post_attention_layernorm",
                "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj",
                "v_proj": "self_attn.v_proj", "o_proj": "self_attn.o_proj",
                "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
                "down_proj": "mlp.down_proj"}.items()})
        pools = [(np.zeros((ns + W, kvd), np.uint16), np.zeros((ns + W, kvd), np.uint16))
                 for _ in range(2)]
        emb = bits(tensors["model.embed_tokens.weight"])
        fnorm = bits(tensors["model.norm.weight"])
        head = bits(tensors["lm_head.weight"])
        ids = np.random.default_rng(2).integers(0, cfg["vocab_size"], 20).astype(np.int32)
        pos = 0
        for step in range(3):
            x = emb[ids]
            for Lw, (kp_, vp_) in zip(Ls, pools):
                x = O.transformer_layer(x, Lw, kp_, vp_, pos, dict(cfg, n_sink=ns, window=W), 0)
            logits = O.linear(O.rmsnorm(x[-1:], fnorm, 0, cfg["rms_norm_eps"]), head, 0, "f32")[0]
            tok = int(model.step(torch.from_numpy(ids).to(dev), pos).item())
            comm.wait()
            ob.device_check()
            assert logits[tok] >= logits.max() - 0.02 * np.abs(logits).max(), (rank, step)
            toks = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(toks, torch.tensor([tok]))
            assert all(int(t_) == tok for t_ in toks), "ranks picked different tokens"
            pos += len(ids)
            ids = np.array([tok], dtype=np.int32)
        torch.cuda.synchronize()
        del model
        comm.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report, never hang the parent
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_layer(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, msg = q.get(timeout=300)
        results[r] = msg
    for p in procs:
        p.join(timeout=120)
    assert all(m == "ok" for m in results.values()), results
