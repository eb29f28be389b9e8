"""The steps around the projections and the whole layer on the GPU: embedding,
RMSNorm, RoPE and the fused q/k-norm + RoPE + K/V append against the oracle
and the reference's own kernels (oracle/_ref), then DecoderLayer and Decoder
(orininfer_b200.layer) against oracle.transformer_layer, a prefill chunk
followed by decode steps."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from orininfer_b200 import _lib
from orininfer_b200 import kernels as K
from orininfer_b200 import weights as Wt
from orininfer_b200.layer import Decoder, DecoderLayer
from tests._util import TORCH_DT, assert_close, bits, from_bits

pytestmark = pytest.mark.gpu


def rand16(rng, shape, dt, scale=1.0):
    return O.round16((rng.standard_normal(shape) * scale).astype(np.float32), dt)


def dev(a, dt):
    return from_bits(a, TORCH_DT[dt]).cuda()


def close(y, r_bits, dt, what):
    return assert_close(y.float(), from_bits(r_bits, TORCH_DT[dt]).float(), what)


def test_embedding_bit_exact_and_reference():
    rng = np.random.default_rng(0)
    table = rng.integers(0, 65535, (1000, 2048), dtype=np.uint16)
    ids = rng.integers(0, 1000, 37).astype(np.int32)
    dt_ = dev(table, 1)
    di = torch.from_numpy(ids).cuda()
    out = torch.empty((37, 2048), dtype=torch.bfloat16, device="cuda")
    K.embedding(out, dt_, di, 37, 2048)
    ref = torch.empty_like(out)
    O.RefKernels().embedding(ref.data_ptr(), dt_.data_ptr(), di.data_ptr(), 37, 2048)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu()), table[ids])
    assert np.array_equal(bits(ref.cpu()), table[ids])
    # an id outside the table: a zero row, no out-of-bounds read
    di[3] = 5000
    K.embedding(out, dt_, di, 37, 2048)
    torch.cuda.synchronize()
    assert not bits(out.cpu())[3].any()


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("rows,dim", [(1, 2048), (512, 2048), (7, 4096), (3, 100), (256, 64)])
def test_rmsnorm(dt, rows, dim):
    rng = np.random.default_rng(rows + dim)
    x = rand16(rng, (rows, dim), dt)
    w = rand16(rng, (dim,), dt, 0.5)
    out = torch.empty((rows, dim), dtype=TORCH_DT[dt], device="cuda")
    K.rmsnorm(out, dev(x, dt), dev(w, dt), rows, dim, 1e-5)
    K.device_check()
    r = O.rmsnorm(x, w, dt, 1e-5)
    mr, mae, exact = close(out.cpu(), r, dt, "rmsnorm")
    assert exact >= 0.97  # one fp32 sum in another order, then the same products


@pytest.mark.parametrize("rows,dim", [(5, 2048), (64, 128)])
def test_rmsnorm_matches_reference_kernel(rows, dim):
    rng = np.random.default_rng(rows)
    x, w = rand16(rng, (rows, dim), 1), rand16(rng, (dim,), 1, 0.5)
    dx, dw = dev(x, 1), dev(w, 1)
    ref = torch.empty((rows, dim), dtype=torch.bfloat16, device="cuda")
    O.RefKernels().rmsnorm(ref.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, dim, 1e-6)
    out = torch.empty_like(ref)
    _lib.shim("kernels::rmsnorm")(out.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, dim, 1e-6)
    torch.cuda.synchronize()
    r = O.rmsnorm(x, w, 1, 1e-6)
    _, _, exact = close(ref.cpu(), r, 1, "reference rmsnorm vs oracle")
    assert exact >= 0.97
    _, _, exact = close(out.cpu(), bits(ref.cpu()), 1, "kernels::rmsnorm vs reference")
    assert exact >= 0.97


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("S,start,nh,nkv,hd", [(1, 0, 32, 4, 64), (1, 2047, 32, 4, 64),
                                               (300, 100, 32, 8, 128), (5, 9000, 16, 8, 64)])
def test_rope(dt, S, start, nh, nkv, hd):
    rng = np.random.default_rng(S + start)
    q, k = rand16(rng, (S, nh, hd), dt), rand16(rng, (S, nkv, hd), dt)
    dq, dk = dev(q, dt), dev(k, dt)
    K.rope(dq, dk, S, nh, nkv, hd, start, 10000.0)
    K.device_check()
    close(dq.cpu(), O.rope(q, start, 10000.0, dt), dt, "rope q")
    close(dk.cpu(), O.rope(k, start, 10000.0, dt), dt, "rope k")


def test_rope_matches_reference_kernel():
    """The reference's own rope kernel on the same data: the same fp32 angle,
    cosf / sinf and products, so the results are bit-identical or nearly."""
    S, start, nh, nkv, hd, theta = 40, 1000, 32, 4, 64, 10000.0
    rng = np.random.default_rng(1)
    q, k = rand16(rng, (S, nh, hd), 1), rand16(rng, (S, nkv, hd), 1)
    rq, rk = dev(q, 1), dev(k, 1)
    O.RefKernels().rope(rq.data_ptr(), rk.data_ptr(), S, nh, nkv, hd, start, theta)
    oq, ok = dev(q, 1), dev(k, 1)
    _lib.shim("kernels::rope")(oq.data_ptr(), ok.data_ptr(), S, nh, nkv, hd, start, theta)
    torch.cuda.synchronize()
    assert (bits(oq.cpu()) == bits(rq.cpu())).mean() >= 0.999
    assert (bits(ok.cpu()) == bits(rk.cpu())).mean() >= 0.999
    close(rq.cpu(), O.rope(q, start, theta, 1), 1, "reference rope vs oracle")


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("S,start,nh,nkv,hd,ns,W", [
    (1, 3000, 32, 4, 64, 4, 1024),
    (64, 0, 32, 4, 64, 4, 1024),
    (18, 20, 16, 8, 128, 2, 16),   # more window positions than slots: later token kept
])
def test_qkv_rope_append(dt, qk_norm, S, start, nh, nkv, hd, ns, W):
    rng = np.random.default_rng(S * 3 + start)
    QD, KVD = nh * hd, nkv * hd
    qkv = rand16(rng, (S, QD + 2 * KVD), dt)
    qn = rand16(rng, (hd,), dt, 0.5) if qk_norm else None
    kn = rand16(rng, (hd,), dt, 0.5) if qk_norm else None
    kp = rand16(rng, (ns + W, KVD), dt)
    vp = rand16(rng, (ns + W, KVD), dt)
    dk, dv = dev(kp, dt), dev(vp, dt)
    q_out = torch.empty((S, QD), dtype=TORCH_DT[dt], device="cuda")
    K.qkv_rope_append(q_out, dev(qkv, dt), dk, dv, S, start, nh, nkv, hd, 10000.0, ns, W,
                      q_norm=dev(qn, dt) if qk_norm else None,
                      k_norm=dev(kn, dt) if qk_norm else None, eps=1e-6)
    K.device_check()
    q, k, v = qkv[:, :QD], qkv[:, QD:QD + KVD], qkv[:, QD + KVD:]
    if qk_norm:
        q = O.rmsnorm(q.reshape(-1, hd), qn, dt, 1e-6)
        k = O.rmsnorm(k.reshape(-1, hd), kn, dt, 1e-6)
    rq = O.rope(q.reshape(S, nh, hd), start, 10000.0, dt)
    rk = O.rope(k.reshape(S, nkv, hd), start, 10000.0, dt)
    O.kv_append(kp, vp, rk.reshape(S, KVD), np.ascontiguousarray(v), start, ns, W)
    close(q_out.cpu(), rq.reshape(S, QD), dt, "q")
    close(dk.cpu(), kp, dt, "k pool")
    assert np.array_equal(bits(dv.cpu()), vp)  # v is copied, never rounded


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("M", [1, 5, 16, 32])
@pytest.mark.parametrize("N,Kd,epi", [(2560, 2048, "none"), (5632, 2048, "swiglu"),
                                      (100, 72, "none"), (512, 4096, "none")])
def test_linear_rmsnorm_equals_norm_then_linear(dt, M, N, Kd, epi):
    """The norm folded into the weight stream gives what orin_rmsnorm then
    orin_linear give (same per-row sum, same rounding of the normed row), and
    matches the oracle."""
    rng = np.random.default_rng(M * 7 + Kd)
    x = rand16(rng, (M, Kd), dt)
    nw = rand16(rng, (Kd,), dt, 0.5)
    w = rand16(rng, (2 * N if epi == "swiglu" else N, Kd), dt, 0.02)
    dx, dn, dw = dev(x, dt), dev(nw, dt), dev(w, dt)
    fused = torch.empty((M, N), dtype=TORCH_DT[dt], device="cuda")
    K.linear_rmsnorm(fused, dx, dw, dn, 1e-5, epilogue=epi)
    xn = torch.empty_like(dx)
    K.rmsnorm(xn, dx, dn, M, Kd, 1e-5)
    plain = torch.empty_like(fused)
    K.linear_into(plain, xn, dw, epilogue=epi, algo="gemv")
    K.device_check()
    assert (bits(fused.cpu()) == bits(plain.cpu())).mean() >= 0.99
    r = O.linear(O.rmsnorm(x, nw, dt, 1e-5), w, dt, epi)
    close(fused.cpu(), r, dt, f"linear_rmsnorm M={M} N={N} K={Kd} {epi}")


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("batch,S,start,ns,W", [
    (1, 1, 2, 4, 1024),      # a sink position
    (1, 1, 700, 4, 1024),    # inside the window
    (1, 1, 3000, 4, 1024),   # the ring has wrapped
    (4, 1, 1500, 4, 1024),   # batched decode: one token of each sequence
    (16, 1, 1029, 4, 1024),  # batch 16 at the first wrapped slot
    (1, 5, 1020, 4, 1024),   # a few tokens across the wrap
    (1, 16, 40, 8, 8),       # tokens of one call sharing ring slots (the later kept)
    (2, 8, 21, 4, 16),       # two sequences of 8 tokens each
])
@pytest.mark.parametrize("shape", [dict(nh=32, nkv=4, hd=64, H=2048),
                                   dict(nh=8, nkv=2, hd=128, H=512)])
def test_linear_rope_append_equals_linear_then_rope_append(dt, batch, S, start, ns, W, shape):
    """RoPE and the K/V append in the q/k/v weight stream's epilogue give bit
    for bit what the projection then orin_qkv_rope_append give: q and both
    pools (which start with random contents), for every position kind."""
    nh, nkv, hd, H = shape["nh"], shape["nkv"], shape["hd"], shape["H"]
    rng = np.random.default_rng(batch * 1000 + S * 10 + start + hd)
    M = batch * S
    rows = (nh + 2 * nkv) * hd
    x = dev(rand16(rng, (M, H), dt), dt)
    w = dev(rand16(rng, (rows, H), dt, 0.05), dt)
    pools = dev(rand16(rng, (2, batch, ns + W, nkv * hd), dt), dt)
    k1, v1 = pools[0].clone(), pools[1].clone()
    k2, v2 = pools[0].clone(), pools[1].clone()
    q1 = torch.empty((M, nh, hd), dtype=TORCH_DT[dt], device="cuda")
    q2 = torch.empty_like(q1)
    K.linear_rope_append(q1, x, w, k1, v1, S, start, nh, nkv, hd, 10000.0, ns, W)
    qkv = torch.empty((M, rows), dtype=TORCH_DT[dt], device="cuda")
    K.linear_into(qkv, x, w, algo="gemv")
    K.qkv_rope_append_batch(q2, qkv, k2, v2, S, start, nh, nkv, hd, 10000.0, ns, W)
    K.device_check()
    what = f"batch={batch} S={S} start={start} n_sink={ns} W={W} {shape} dt={dt}"
    assert np.array_equal(bits(q1.cpu()), bits(q2.cpu())), what
    assert np.array_equal(bits(k1.cpu()), bits(k2.cpu())), what
    assert np.array_equal(bits(v1.cpu()), bits(v2.cpu())), what


@pytest.mark.parametrize("M", [1, 3])
def test_lm_head_argmax_with_folded_norm(M):
    dt = 1
    rng = np.random.default_rng(M)
    h = rand16(rng, (M, 2048), dt)
    nw = rand16(rng, (2048,), dt, 0.5)
    w = rand16(rng, (32000, 2048), dt, 0.02)
    dh, dn, dw = dev(h, dt), dev(nw, dt), dev(w, dt)
    tok = K.lm_head_argmax(dh, dw, norm=dn, eps=1e-5)
    hn = torch.empty_like(dh)
    K.rmsnorm(hn, dh, dn, M, 2048, 1e-5)
    tok2 = K.lm_head_argmax(hn, dw)
    K.device_check()
    assert tok.cpu().tolist() == tok2.cpu().tolist()
    r = O.lm_head_argmax(O.rmsnorm(h, nw, dt, 1e-5), w, dt)
    assert tok.cpu().tolist() == r.tolist()


SMALL = dict(hidden_size=512, intermediate_size=1408, num_attention_heads=8,
             num_key_value_heads=2, head_dim=64, vocab_size=3000, rms_norm_eps=1e-5,
             rope_theta=10000.0)


def layer_bits(tensors, i, dt):
    p = f"model.layers.{i}"
    names = {"input_layernorm": "input_layernorm", "post_attention_layernorm":
             "post_attention_layernorm", "q_proj": "self_attn.q_proj", "k_proj":
             "self_attn.k_proj", "v_proj": "self_attn.v_proj", "o_proj": "self_attn.o_proj",
             "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm", "gate_proj":
             "mlp.gate_proj", "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}
    return {k: bits(tensors[f"{p}.{v}.weight"]) for k, v in names.items()}


@pytest.mark.parametrize("fold_norm", [False, True])
@pytest.mark.parametrize("dims,qk_norm,dt", [
    (dict(), False, 0),                # TinyLlama layer
    (SMALL, True, 1),                  # Qwen3-style q/k norm, bf16
])
def test_decoder_layer_matches_oracle(dims, qk_norm, dt, fold_norm):
    """A 100-token prefill then 3 decode tokens through one layer (the decode
    tokens with and without the norms folded into the weight stream)."""
    torch_dt = TORCH_DT[dt]
    tensors, cfg = Wt.synthetic_model(1, seed=3, dtype=torch_dt, **dims)
    if qk_norm:  # non-trivial norm weights
        g = torch.Generator().manual_seed(9)
        for n in ("q_norm", "k_norm"):
            t = tensors[f"model.layers.0.self_attn.{n}.weight"]
            tensors[f"model.layers.0.self_attn.{n}.weight"] = \
                (1 + 0.3 * torch.randn(t.shape, generator=g)).to(torch_dt)
    ns, W = 4, 64
    layer = DecoderLayer(Wt.layer_for_device(tensors, 0, cfg, "cuda"), cfg, n_sink=ns, window=W,
                         max_tokens=ns + W, qk_norm=qk_norm, fold_norm=fold_norm)
    L = layer_bits(tensors, 0, dt)
    if not qk_norm:
        L["q_norm"] = L["k_norm"] = None
    ocfg = dict(cfg, n_sink=ns, window=W)
    KVD = cfg["num_key_value_heads"] * cfg["head_dim"]
    kp = np.zeros((ns + W, KVD), dtype=np.uint16)
    vp = np.zeros_like(kp)
    rng = np.random.default_rng(4)
    pos = 0
    for S in (68, 32, 1, 1, 1):
        x = rand16(rng, (S, cfg["hidden_size"]), dt)
        y = layer.forward(dev(x, dt), pos)
        K.device_check()
        r = O.transformer_layer(x, L, kp, vp, pos, ocfg, dt)
        close(y.cpu(), r, dt, f"layer at {pos} (+{S})")
        pos += S


@pytest.mark.parametrize("fold_norm", [False, True])
def test_decoder_greedy_step(fold_norm):
    """Two layers, prefill then decode: each token the library picks has an
    oracle logit within the tolerance of the oracle's best."""
    dt = 1
    tensors, cfg = Wt.synthetic_model(2, seed=5, dtype=torch.bfloat16, **SMALL)
    ns, W = 4, 60
    model = Decoder(tensors, cfg, "cuda", n_sink=ns, window=W, max_tokens=ns + W,
                    fold_norm=fold_norm)
    Ls = [layer_bits(tensors, i, dt) for i in range(2)]
    for L in Ls:
        L["q_norm"] = L["k_norm"] = None
    ocfg = dict(cfg, n_sink=ns, window=W)
    KVD = cfg["num_key_value_heads"] * cfg["head_dim"]
    pools = [(np.zeros((ns + W, KVD), np.uint16), np.zeros((ns + W, KVD), np.uint16))
             for _ in range(2)]
    emb = bits(tensors["model.embed_tokens.weight"])
    fnorm = bits(tensors["model.norm.weight"])
    head = bits(tensors["lm_head.weight"])
    ids = np.random.default_rng(2).integers(0, cfg["vocab_size"], 30).astype(np.int32)
    pos = 0
    for step in range(4):
        x = emb[ids]
        for L, (kp, vp) in zip(Ls, pools):
            x = O.transformer_layer(x, L, kp, vp, pos, ocfg, dt)
        h = O.rmsnorm(x[-1:], fnorm, dt, cfg["rms_norm_eps"])
        logits = O.linear(h, head, dt, "f32")[0]
        tok = int(model.step(torch.from_numpy(ids).cuda(), pos).item())
        assert logits[tok] >= logits.max() - 0.02 * np.abs(logits).max(), step
        pos += len(ids)
        ids = np.array([tok], dtype=np.int32)
