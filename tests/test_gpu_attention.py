"""Sink + sliding-window GQA attention and the K/V scatter on the GPU, through
the C ABI, against the oracle (oracle.attention, oracle.kv_append); the oracle
itself pinned to the reference's own attention kernel (kernels/attention.cu,
built from its sources into oracle/_ref) on the same inputs.

Tolerance: the attention output is one 16-bit rounding of fp32 sums on both
sides; the kernel rounds the softmax weights to 16 bits for the tensor-core
P.V product, so the bar is the GEMM one (max relative error 1e-2 of the
largest output, mean absolute error 1e-3), not bit-identity."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from orininfer_b200 import _lib
from orininfer_b200 import kernels as K
from tests._util import TORCH_DT, assert_close, bits, from_bits

pytestmark = pytest.mark.gpu

TINY = dict(nh=32, nkv=4, hd=64)     # TinyLlama attention
LLAMA3 = dict(nh=32, nkv=8, hd=128)  # Llama-3-8B attention


def rand16(rng, shape, dt):
    return O.round16(rng.standard_normal(shape).astype(np.float32), dt)


def dev(a, dt):
    return from_bits(a, TORCH_DT[dt]).cuda()


def inputs(seed, S, nh, nkv, hd, ns, W, dt):
    rng = np.random.default_rng(seed)
    return (rand16(rng, (S, nh, hd), dt), rand16(rng, (ns + W, nkv, hd), dt),
            rand16(rng, (ns + W, nkv, hd), dt))


def ours(q, kp, vp, S, C, nh, nkv, hd, ns, W, dt, **kw):
    out = torch.empty((S, nh, hd), dtype=TORCH_DT[dt], device="cuda")
    K.attention(out, dev(q, dt), dev(kp, dt), dev(vp, dt), S, C, nh, nkv, hd, hd ** -0.5, ns, W,
                **kw)
    K.device_check()
    return out.cpu()


def check(y, r_bits, dt, what):
    assert_close(y.float(), from_bits(r_bits, TORCH_DT[dt]).float(), what)


CASES = [
    # (S, C, shape, n_sink, W): decode at several fill levels, prefill chunks
    (1, 1, TINY, 4, 1024),
    (1, 4, TINY, 4, 1024),
    (1, 5, TINY, 4, 1024),
    (1, 700, TINY, 4, 1024),
    (1, 1028, TINY, 4, 1024),
    (1, 1029, TINY, 4, 1024),
    (1, 5000, TINY, 4, 1024),
    (4, 2100, TINY, 4, 1024),
    (1028, 1028, TINY, 4, 1024),   # first prefill chunk of a 2048-token prompt
    (1020, 2048, TINY, 4, 1024),   # second chunk: wraps the ring onto itself
    (1, 3000, LLAMA3, 4, 1024),
    (300, 300, LLAMA3, 4, 1024),
    (77, 600, dict(nh=8, nkv=2, hd=64), 4, 80),     # many ring wraps, small window
    (37, 37, dict(nh=16, nkv=16, hd=128), 0, 16),   # MHA, no sink
    (5, 1000, dict(nh=64, nkv=1, hd=64), 4, 200),   # one KV head for 64 query heads
    (3, 50, dict(nh=128, nkv=1, hd=64), 4, 32),     # group larger than a row block
    (2, 9, dict(nh=6, nkv=2, hd=64), 4, 1024),      # group of 3 (rows left over)
]


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("S,C,shape,ns,W", CASES)
def test_attention_matches_oracle(dt, S, C, shape, ns, W):
    nh, nkv, hd = shape["nh"], shape["nkv"], shape["hd"]
    q, kp, vp = inputs(S * 7 + C, S, nh, nkv, hd, ns, W, dt)
    r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    check(ours(q, kp, vp, S, C, nh, nkv, hd, ns, W, dt), r, dt, f"attention S={S} C={C}")


@pytest.mark.parametrize("ws", ["none", "short", "full"])
def test_attention_split_keys_agree(ws):
    """Decode with the keys split across CTAs (full workspace), fewer splits
    (a short one) and none: all three match the oracle."""
    dt, S, C, ns, W = 1, 1, 4000, 4, 1024
    nh, nkv, hd = TINY["nh"], TINY["nkv"], TINY["hd"]
    q, kp, vp = inputs(11, S, nh, nkv, hd, ns, W, dt)
    r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    need = K.attention_workspace_bytes(S, C, nh, nkv, hd, ns, W)
    assert need > 0
    kw = {"none": dict(split=False),
          "short": dict(workspace=torch.zeros(need // 3, dtype=torch.uint8, device="cuda")),
          "full": dict()}[ws]
    check(ours(q, kp, vp, S, C, nh, nkv, hd, ns, W, dt, **kw), r, dt, f"split {ws}")


@pytest.mark.parametrize("S,C,shape,ns,W", [
    (1, 1, TINY, 4, 1024),
    (1, 1029, TINY, 4, 1024),
    (1, 5000, TINY, 4, 1024),
    (64, 1028, TINY, 4, 1024),
    (1020, 2048, TINY, 4, 1024),
    (1, 3000, LLAMA3, 4, 1024),
    (33, 300, dict(nh=8, nkv=2, hd=64), 4, 80),
])
def test_oracle_matches_reference_attention_kernel(S, C, shape, ns, W):
    """Pin: the reference's own kernel (bf16) on the same pools and queries."""
    ref = O.RefKernels()
    dt = 1
    nh, nkv, hd = shape["nh"], shape["nkv"], shape["hd"]
    q, kp, vp = inputs(S * 13 + C, S, nh, nkv, hd, ns, W, dt)
    dq, dk, dv = dev(q, dt), dev(kp, dt), dev(vp, dt)
    out = torch.zeros((S, nh, hd), dtype=torch.bfloat16, device="cuda")
    ref.attention(out.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), S, C, nh, nkv, hd,
                  hd ** -0.5, ns, W)
    ref.sync()
    r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    # same fp32 arithmetic on both sides (fp64 in the oracle): one-unit
    # rounding flips at most
    _, _, exact = assert_close(out.cpu().float(), from_bits(r, torch.bfloat16).float(),
                               "reference kernel vs oracle", max_rel=4e-3, mae=2e-4)
    assert exact >= 0.95
    # and this library against the reference kernel directly
    mine = ours(q, kp, vp, S, C, nh, nkv, hd, ns, W, dt)
    check(mine, bits(out.cpu()), dt, "ours vs reference")
    if C > 64:
        # this library rounds the softmax weights to 16 bits for the tensor
        # cores and the reference does not: two implementations are compared
        assert (bits(mine) != bits(out.cpu())).any()


@pytest.mark.parametrize("start,S,ns,W,kv_dim", [
    (0, 1028, 4, 1024, 256),    # first chunk: sinks + a full window
    (1028, 1020, 4, 1024, 256),  # second chunk, wraps
    (5000, 1, 4, 1024, 256),    # one decode token
    (2, 1028, 4, 1024, 256),    # more window positions than slots: later token kept
    (3, 18, 2, 16, 12),         # rows not a multiple of 16 bytes (scalar copies), slot reuse
])
def test_kv_append_bit_exact(start, S, ns, W, kv_dim):
    rng = np.random.default_rng(start + S)
    kp = rng.integers(0, 65535, (ns + W, kv_dim), dtype=np.uint16)
    vp = rng.integers(0, 65535, (ns + W, kv_dim), dtype=np.uint16)
    ks = rng.integers(0, 65535, (S, kv_dim), dtype=np.uint16)
    vs = rng.integers(0, 65535, (S, kv_dim), dtype=np.uint16)
    dk, dv = dev(kp, 0), dev(vp, 0)
    K.kv_append(dk, dv, dev(ks, 0), dev(vs, 0), S, start, ns, W)
    K.device_check()
    O.kv_append(kp, vp, ks, vs, start, ns, W)
    assert np.array_equal(bits(dk.cpu()), kp)
    assert np.array_equal(bits(dv.cpu()), vp)


@pytest.mark.parametrize("dt", [0, 1])
def test_prefill_chunks_then_decode_as_the_reference_runs_them(dt):
    """The reference's per-layer order (src/model.cu:75-84; chunks from
    src/engine.cpp:67-81): append the call's K/V, then attend.  A 2048-token
    prompt in chunks of 1028 and 1020, then 3 decode tokens."""
    nh, nkv, hd, ns, W = TINY["nh"], TINY["nkv"], TINY["hd"], 4, 1024
    rng = np.random.default_rng(5)
    kp = np.zeros((ns + W, nkv * hd), dtype=np.uint16)
    vp = np.zeros_like(kp)
    dk, dv = dev(kp, dt), dev(vp, dt)
    pos = 0
    for S in (1028, 1020, 1, 1, 1):
        q = rand16(rng, (S, nh, hd), dt)
        ks = rand16(rng, (S, nkv * hd), dt)
        vs = rand16(rng, (S, nkv * hd), dt)
        O.kv_append(kp, vp, ks, vs, pos, ns, W)
        K.kv_append(dk, dv, dev(ks, dt), dev(vs, dt), S, pos, ns, W)
        C = pos + S
        r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
        out = torch.empty((S, nh, hd), dtype=TORCH_DT[dt], device="cuda")
        K.attention(out, dev(q, dt), dk, dv, S, C, nh, nkv, hd, hd ** -0.5, ns, W)
        K.device_check()
        check(out.cpu(), r, dt, f"chunk at {pos} (+{S})")
        pos = C
    assert np.array_equal(bits(dk.cpu()), kp)


def test_reference_signature_entry_point():
    """kernels::attention (include/kernels.h:67-80) from liborin_b200.so:
    bf16, default stream, split partials in the library's static array."""
    S, C, ns, W = 1, 3000, 4, 1024
    nh, nkv, hd = TINY["nh"], TINY["nkv"], TINY["hd"]
    q, kp, vp = inputs(3, S, nh, nkv, hd, ns, W, 1)
    dq, dk, dv = dev(q, 1), dev(kp, 1), dev(vp, 1)
    out = torch.zeros((S, nh, hd), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    _lib.shim("kernels::attention")(out.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                    S, C, nh, nkv, hd, hd ** -0.5, ns, W)
    torch.cuda.synchronize()
    r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, 1)
    check(out.cpu(), r, 1, "kernels::attention")


def test_attention_in_a_cuda_graph():
    """Decode attention (split keys + combine) captured once and replayed."""
    dt, S, C, ns, W = 0, 1, 2500, 4, 1024
    nh, nkv, hd = TINY["nh"], TINY["nkv"], TINY["hd"]
    q, kp, vp = inputs(17, S, nh, nkv, hd, ns, W, dt)
    dq, dk, dv = dev(q, dt), dev(kp, dt), dev(vp, dt)
    out = torch.empty((S, nh, hd), dtype=TORCH_DT[dt], device="cuda")
    ws = torch.zeros(K.attention_workspace_bytes(S, C, nh, nkv, hd, ns, W), dtype=torch.uint8,
                     device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        K.attention(out, dq, dk, dv, S, C, nh, nkv, hd, hd ** -0.5, ns, W, workspace=ws)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        K.attention(out, dq, dk, dv, S, C, nh, nkv, hd, hd ** -0.5, ns, W, workspace=ws)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    r = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    check(out.cpu(), r, dt, "graph replay")


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("C,shape", [(1029, TINY), (2048 + 7, TINY), (300, LLAMA3), (3, TINY)])
def test_attention_batch_equals_per_sequence_calls(dt, C, shape):
    """orin_attention_batch over 5 sequences with their own pools: every
    sequence's output bit-identical to its own orin_attention call (same key
    splits and summation order), and within the bar of the oracle."""
    B, ns, W = 5, 4, 1024
    nh, nkv, hd = shape["nh"], shape["nkv"], shape["hd"]
    rng = np.random.default_rng(77 + C)
    q = [rand16(rng, (1, nh, hd), dt) for _ in range(B)]
    kp = [rand16(rng, (ns + W, nkv, hd), dt) for _ in range(B)]
    vp = [rand16(rng, (ns + W, nkv, hd), dt) for _ in range(B)]
    qb = torch.stack([dev(a, dt) for a in q])
    kb = torch.stack([dev(a, dt) for a in kp])
    vb = torch.stack([dev(a, dt) for a in vp])
    out = torch.empty((B, 1, nh, hd), dtype=TORCH_DT[dt], device="cuda")
    K.attention_batch(out, qb, kb, vb, 1, C, nh, nkv, hd, hd ** -0.5, ns, W)
    K.device_check()
    for b in range(B):
        single = ours(q[b], kp[b], vp[b], 1, C, nh, nkv, hd, ns, W, dt)
        assert torch.equal(out[b].cpu().view(torch.int16), single.view(torch.int16)), b
        r = O.attention(q[b], kp[b], vp[b], 1, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
        check(out[b].cpu(), r, dt, f"batch seq {b}")


@pytest.mark.parametrize("dt", [0, 1])
def test_qkv_rope_append_batch_equals_per_sequence_calls(dt):
    """orin_qkv_rope_append_batch: 6 sequences' decode rows at one position,
    each appended to its own pools; q rows and every pool bit-identical to
    per-sequence orin_qkv_rope_append calls."""
    B, nh, nkv, hd, ns, W, pos = 6, 32, 4, 64, 4, 1024, 1500
    tdt = TORCH_DT[dt]
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn((B, (nh + 2 * nkv) * hd), generator=g).to(tdt).cuda()
    kb = torch.randn((B, ns + W, nkv * hd), generator=g).to(tdt).cuda()
    vb = torch.randn((B, ns + W, nkv * hd), generator=g).to(tdt).cuda()
    k1, v1 = kb.clone(), vb.clone()
    qo = torch.empty((B, nh * hd), dtype=tdt, device="cuda")
    K.qkv_rope_append_batch(qo, qkv, kb, vb, 1, pos, nh, nkv, hd, 10000.0, ns, W)
    q1 = torch.empty((1, nh * hd), dtype=tdt, device="cuda")
    for b in range(B):
        K.qkv_rope_append(q1, qkv[b:b + 1], k1[b], v1[b], 1, pos, nh, nkv, hd, 10000.0, ns, W)
        assert torch.equal(qo[b:b + 1].view(torch.int16), q1.view(torch.int16)), b
    K.device_check()
    assert torch.equal(kb.view(torch.int16), k1.view(torch.int16))
    assert torch.equal(vb.view(torch.int16), v1.view(torch.int16))
