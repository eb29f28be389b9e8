"""The attention oracle (CPU only): the vectorised restatement against the
literal one that follows the reference kernel's ring-offset arithmetic
(kernels/attention.cu:41-55), the K/V scatter, and the reference's
scatter-before-attend behaviour when a chunk wraps the ring (src/model.cu:75-84)."""
import numpy as np
import pytest

from oracle import oracle as O

F16, BF16 = O.F16, O.BF16


def rand16(rng, shape, dt, scale=1.0):
    return O.round16((rng.standard_normal(shape) * scale).astype(np.float32), dt)


@pytest.mark.parametrize("dt", [F16, BF16])
@pytest.mark.parametrize("S,C,nh,nkv,hd,ns,W", [
    (1, 1, 4, 2, 64, 4, 16),      # first token: sink only
    (3, 3, 4, 1, 64, 4, 16),      # prefill shorter than the sink
    (20, 20, 8, 2, 64, 4, 16),    # prefill past the window
    (1, 50, 8, 2, 64, 4, 16),     # decode with a wrapped ring
    (7, 61, 4, 4, 64, 0, 8),      # no sink, MHA
    (19, 40, 4, 2, 128, 3, 16),   # chunk continuing a wrapped ring
    (12, 12, 8, 8, 64, 2, 10),    # chunk of exactly n_sink + W
])
def test_vectorised_matches_literal(dt, S, C, nh, nkv, hd, ns, W):
    rng = np.random.default_rng(S * 1000 + C)
    q = rand16(rng, (S, nh, hd), dt)
    kp = rand16(rng, (ns + W, nkv, hd), dt)
    vp = rand16(rng, (ns + W, nkv, hd), dt)
    a = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    b = O.attention_literal(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    fa, fb = O.widen(a, dt), O.widen(b, dt)
    # fp64 against fp32: only final roundings may differ, by one unit
    if dt == F16:
        ulp = np.maximum(np.abs(np.spacing(fa.astype(np.float16))),
                         np.abs(np.spacing(fb.astype(np.float16)))).astype(np.float32)
    else:
        ulp = np.maximum(np.abs(fa), np.abs(fb)) * 2.0 ** -7
    assert np.all(np.abs(fa - fb) <= ulp)
    assert (a == b).mean() >= 0.99


def test_ring_slots():
    assert list(O.ring_slot(range(10), 4, 3)) == [0, 1, 2, 3, 4, 5, 6, 4, 5, 6]
    assert list(O.ring_slot(range(5), 0, 2)) == [0, 1, 0, 1, 0]


def test_kv_append_slots_and_later_token_wins():
    ns, W, D = 2, 4, 3
    kp = np.zeros((ns + W, D), dtype=np.int64)
    vp = np.zeros_like(kp)
    src = np.arange(6 * D).reshape(6, D)
    # positions 1..6: 1 -> slot 1, 2..5 -> 2..5, 6 -> slot 2 (overwrites position 2)
    O.kv_append(kp, vp, src, -src, 1, ns, W)
    assert (kp[1] == src[0]).all() and (kp[2] == src[5]).all() and (kp[5] == src[4]).all()
    assert (vp[2] == -src[5]).all()
    assert (kp[0] == 0).all()
    with pytest.raises(ValueError):
        O.kv_append(kp, vp, np.zeros((7, D)), np.zeros((7, D)), 0, ns, W)


def test_wrapped_chunk_reads_its_own_later_tokens():
    """Prefill 10 positions (2 sinks + window 8), then a chunk of 8 more: the
    chunk's first query (position 10) sees window positions 3..10, but slots
    3..9 already hold positions 11..17 of the same chunk, and that is what the
    reference (and the oracle) reads."""
    dt, ns, W, hd = F16, 2, 8, 64
    rng = np.random.default_rng(7)
    k_all = rand16(rng, (18, 1, hd), dt)
    v_all = rand16(rng, (18, 1, hd), dt)
    q = rand16(rng, (8, 1, hd), dt)
    kp = np.zeros((ns + W, 1, hd), dtype=np.uint16)
    vp = np.zeros_like(kp)
    O.kv_append(kp, vp, k_all[:10], v_all[:10], 0, ns, W)
    O.kv_append(kp, vp, k_all[10:], v_all[10:], 10, ns, W)
    out = O.widen(O.attention(q, kp, vp, 8, 18, 1, 1, hd, hd ** -0.5, ns, W, dt), dt)

    def direct(qrow, positions):
        kk = O.widen(k_all[positions, 0], dt).astype(np.float64)
        vv = O.widen(v_all[positions, 0], dt).astype(np.float64)
        s = kk @ O.widen(qrow, dt).astype(np.float64) * hd ** -0.5
        e = np.exp(s - s.max())
        return (e @ vv) / e.sum()

    # slots 0,1 = positions 0,1; slot 2 = position 10; slots 3..9 = positions 11..17
    as_stored = direct(q[0, 0], [0, 1, 10, 11, 12, 13, 14, 15, 16, 17])
    causal = direct(q[0, 0], [0, 1, 3, 4, 5, 6, 7, 8, 9, 10])
    assert np.abs(out[0, 0] - as_stored).max() < 2e-3
    assert np.abs(out[0, 0] - causal).max() > 1e-2
    # the chunk's last query sees exactly the positions it should
    last = direct(q[7, 0], [0, 1, 10, 11, 12, 13, 14, 15, 16, 17])
    assert np.abs(out[7, 0] - last).max() < 2e-3


@pytest.mark.parametrize("dt", [F16, BF16])
def test_constant_values_come_back_exactly(dt):
    """Softmax weights sum to one: if every V row is the same vector, every
    output is that vector (one rounding of an exact value)."""
    rng = np.random.default_rng(1)
    S, C, nh, nkv, hd, ns, W = 9, 300, 8, 2, 64, 4, 100
    q = rand16(rng, (S, nh, hd), dt)
    kp = rand16(rng, (ns + W, nkv, hd), dt)
    row = rand16(rng, (1, 1, hd), dt)
    vp = np.broadcast_to(row, (ns + W, nkv, hd)).copy()
    out = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    assert np.array_equal(out, np.broadcast_to(row, (S, nh, hd)))


@pytest.mark.parametrize("dt", [F16, BF16])
def test_no_sink_and_a_long_window_is_causal_attention(dt):
    """With n_sink = 0 and a window longer than the sequence nothing is
    evicted: plain causal softmax attention over positions 0..ap."""
    rng = np.random.default_rng(2)
    S, nh, hd = 20, 4, 64
    q = rand16(rng, (S, nh, hd), dt)
    k = rand16(rng, (S, nh, hd), dt)
    v = rand16(rng, (S, nh, hd), dt)
    W = 64
    kp = np.zeros((W, nh, hd), np.uint16)
    vp = np.zeros_like(kp)
    O.kv_append(kp.reshape(W, -1), vp.reshape(W, -1), k.reshape(S, -1), v.reshape(S, -1), 0, 0, W)
    out = O.widen(O.attention(q, kp, vp, S, S, nh, nh, hd, hd ** -0.5, 0, W, dt), dt)
    qf, kf, vf = (O.widen(a, dt).astype(np.float64) for a in (q, k, v))
    s = np.einsum("thd,uhd->htu", qf, kf) * hd ** -0.5
    s = np.where(np.tril(np.ones((S, S), bool))[None], s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    ref = np.einsum("htu,uhd->thd", p / p.sum(-1, keepdims=True), vf)
    assert np.abs(out - ref).max() <= 2 ** -7 * np.abs(ref).max()


def test_grouped_query_heads_equal_repeated_kv_heads():
    """G query heads sharing a KV head give what G copies of that KV head would."""
    dt = BF16
    rng = np.random.default_rng(3)
    S, C, nh, nkv, hd, ns, W = 5, 70, 8, 2, 64, 4, 32
    q = rand16(rng, (S, nh, hd), dt)
    kp = rand16(rng, (ns + W, nkv, hd), dt)
    vp = rand16(rng, (ns + W, nkv, hd), dt)
    gqa = O.attention(q, kp, vp, S, C, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    G = nh // nkv
    mha = O.attention(q, np.repeat(kp, G, axis=1), np.repeat(vp, G, axis=1), S, C, nh, nh, hd,
                      hd ** -0.5, ns, W, dt)
    assert np.array_equal(gqa, mha)
