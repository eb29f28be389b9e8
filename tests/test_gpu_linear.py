"""Parity of the CUDA linear-layer kernels with the CPU oracle (B200 only).

Every case: seeded 16-bit inputs, the kernel through the C ABI (via the
Python mirror), the oracle on the same bits, and the parity bar of
tests/_util.py (max relative error <= 1e-2, mean absolute error <= 1e-3).
"""
import numpy as np
import pytest
import torch

import orininfer_b200 as ob
from orininfer_b200 import _lib
from oracle import oracle as orc
from tests._util import EXACT_MIN, TORCH_DT, assert_close, bits, elem_max_for, from_bits, seeded

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def run_case(M, N, K, dt, epi, algo="auto", seed=0, check_rows=None):
    tdt = TORCH_DT[dt]
    wrows = 2 * N if epi == "swiglu" else N
    x = seeded((M, K), seed + 1, 1.0, tdt)
    w = seeded((wrows, K), seed + 2, 0.02, tdt)
    res = seeded((M, N), seed + 3, 1.0, tdt) if epi == "residual" else None
    y = ob.linear(x.to(DEV), w.to(DEV), epilogue=epi,
                  residual=res.to(DEV) if res is not None else None, algo=algo)
    ob.device_check()
    y = y.cpu()
    rows = np.arange(M) if check_rows is None else check_rows
    xr = x[rows]
    rr = bits(res[rows]) if res is not None else None
    ref = orc.linear(bits(xr), bits(w), dt, epi, rr)
    if epi in ("f32", "f32_partial"):
        ref_t = torch.from_numpy(ref)
    else:
        ref_t = from_bits(ref, tdt).float()
    # the elementwise relative error is asserted where no residual add cancels
    assert_close(y[rows].float(), ref_t.float(), f"{algo} {epi} dt={dt} M={M} N={N} K={K}",
                 exact_min=None if epi == "f32_partial" else EXACT_MIN,
                 elem_max=elem_max_for(dt) if epi in ("none", "f32", "swiglu") else None)
    return y


WIDE = [(128, 256, 64), (256, 512, 1024), (200, 300, 136), (65, 1000, 8), (512, 2560, 2048),
        (2048, 5120, 256)]
SKINNY = [(1, 2048, 2048), (1, 128, 64), (3, 200, 520), (16, 384, 2048), (17, 256, 128),
          (32, 2560, 2048), (33, 1024, 1024), (64, 2048, 5632)]


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("M,N,K", WIDE)
def test_wide_none(dt, M, N, K):
    run_case(M, N, K, dt, "none", "wide")


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("M,N,K", SKINNY)
def test_skinny_none(dt, M, N, K):
    run_case(M, N, K, dt, "none", "skinny")


@pytest.mark.parametrize("epi", ["residual", "f32", "f32_partial", "swiglu"])
@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("algo,M,N,K", [("wide", 256, 640, 512), ("wide", 130, 192, 2048),
                                        ("skinny", 1, 704, 2048), ("skinny", 40, 384, 1024)])
def test_epilogues(epi, dt, algo, M, N, K):
    if epi == "swiglu" and N % 64:
        pytest.skip("swiglu needs N % 64 == 0")
    run_case(M, N, K, dt, epi, algo)


GEMV = [(1, 2048, 2048), (1, 200, 520), (3, 384, 72), (8, 2560, 2048), (9, 1024, 5632),
        (16, 256, 8), (5, 4100, 136), (17, 520, 1000), (24, 2048, 2048), (32, 1024, 5632)]


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("M,N,K", GEMV)
def test_gemv_none(dt, M, N, K):
    # decode weight stream: ragged feature groups (N % 16), K not a multiple of
    # the 32-element k-block, K = 8 (one block: seven warps without work), one
    # to four 8-token tiles
    run_case(M, N, K, dt, "none", "gemv")


@pytest.mark.parametrize("epi", ["residual", "f32", "f32_partial", "swiglu"])
@pytest.mark.parametrize("M", [1, 7, 16, 29])
def test_gemv_epilogues(epi, M):
    run_case(M, 384, 1000, 1 if M == 7 else 0, epi, "gemv", seed=M)


def test_gemv_is_the_decode_default():
    for M in (1, 8, 16):
        assert ob.plan_info(M, 2048, 2048)["kernel"] == "gemv"
    assert ob.plan_info(17, 2048, 2048)["kernel"] == "tcgen05-skinny"
    assert ob.plan_info(32, 2048, 2048, algo="gemv")["kernel"] == "gemv"


@pytest.mark.parametrize("epi", ["none", "residual", "swiglu", "f32"])
@pytest.mark.parametrize("M", [1, 24, 64])
@pytest.mark.parametrize("K", [256, 384, 512, 640, 768, 896])
def test_skinny_split_factors(epi, M, K):
    # two 128-row weight tiles and K/128 pairs of 64-wide k-blocks: the
    # planner splits K over K/128 CTAs of a cluster (2..7), each pushing its
    # partial rows to the CTAs that own them
    N = 128 if epi == "swiglu" else 256
    plan = ob.plan_info(M, N, K, torch.float16, epi, "skinny")
    assert plan["split_k"] == K // 128, plan
    run_case(M, N, K, 0, epi, "skinny", seed=K + M)


@pytest.mark.parametrize("epi", ["none", "residual", "swiglu", "f32"])
def test_simt_path_unaligned_k(epi):
    # K % 8 != 0: TMA can't describe the rows; the CUDA-core kernel serves it
    run_case(7, 128, 12, 0, epi, "auto")
    run_case(3, 192, 100, 1, epi, "simt")


def test_residual_in_place():
    """The residual output may alias the residual input (x += o_proj(attn))."""
    M, N, K = 256, 512, 512
    x = seeded((M, K), 5, 1.0)
    w = seeded((N, K), 6, 0.02)
    res = seeded((M, N), 7, 1.0)
    r = res.to(DEV)
    ob.linear_into(r, x.to(DEV), w.to(DEV), epilogue="residual", residual=r)
    ob.device_check()
    ref = orc.linear(bits(x), bits(w), 0, "residual", bits(res))
    assert_close(r.cpu().float(), from_bits(ref, torch.float16).float(), "in-place residual")


def test_output_guard_regions_untouched():
    for algo, (M, N, K) in (("wide", (200, 300, 136)), ("skinny", (5, 200, 64)),
                            ("gemv", (5, 200, 64))):
        guard = 4096
        buf = torch.full((guard + M * N + guard,), 1234.0, dtype=torch.float16, device=DEV)
        out = buf[guard:guard + M * N].view(M, N)
        x = seeded((M, K), 1, 1.0).to(DEV)
        w = seeded((N, K), 2, 0.02).to(DEV)
        ob.linear_into(out, x, w, algo=algo)
        ob.device_check()
        assert (buf[:guard] == 1234.0).all() and (buf[guard + M * N:] == 1234.0).all()


def test_dependent_chain_with_programmatic_launch():
    """A chain of dependent GEMMs back to back (each kernel starts its weight
    loads before the previous one finishes) matches the oracle chain."""
    dims = [512, 1024, 256, 768, 512]
    for M, algo in ((1, "skinny"), (48, "skinny"), (256, "wide"), (1, "gemv"), (12, "gemv")):
        x = seeded((M, dims[0]), 10, 1.0)
        ws = [seeded((dims[i + 1], dims[i]), 20 + i, 0.05) for i in range(len(dims) - 1)]
        h = x.to(DEV)
        for w in ws:
            h = ob.linear(h, w.to(DEV), algo=algo)
        ob.device_check()
        r = bits(x)
        for w in ws:
            r = orc.linear(r, bits(w), 0, "none")
        assert_close(h.cpu().float(), from_bits(r, torch.float16).float(), f"chain {algo} M={M}")


def test_tinyllama_layer_prefill_m512():
    """All four projections of a TinyLlama-shaped layer at M=512, fused epilogues."""
    M, H, IM, KVD = 512, 2048, 5632, 256
    for dt in (0, 1):
        run_case(M, H + 2 * KVD, H, dt, "none", seed=100)      # q/k/v fused
        run_case(M, H, H, dt, "residual", seed=200)            # o_proj + residual
        run_case(M, IM, H, dt, "swiglu", seed=300)             # gate/up + SwiGLU
        run_case(M, H, IM, dt, "residual", seed=400)           # down + residual


def test_llama3_8b_projection_rows_sampled():
    """Llama-3-8B projection at prefill M=4096: oracle on a sample of rows."""
    rows = np.array([0, 1, 127, 128, 2049, 4000, 4095])
    run_case(4096, 6144, 4096, 0, "none", seed=500, check_rows=rows)
    run_case(4096, 4096, 14336, 0, "residual", seed=600, check_rows=rows)


@pytest.mark.parametrize("M", [1, 8, 32, 64])
def test_decode_lm_head_f32(M):
    """LM head at decode: vocab 32000 x 2048, fp32 logits (bf16_to_fp32 folded in)."""
    run_case(M, 32000, 2048, 0, "f32", seed=700 + M)


def _gpu_logits(h, w, dt):
    """The weight-stream kernel's own fp32 logits (F32_OUT: round16 then
    widen), 32 rows at a time — the same accumulation as the fused argmax."""
    rows = [ob.linear(h[r:r + 32], w, epilogue="f32", algo="gemv") for r in range(0, h.shape[0], 32)]
    return torch.cat(rows).cpu().numpy()


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("M", [1, 5, 33])
def test_lm_head_argmax(dt, M):
    """Greedy token per row == the reference sampler's choice over the same
    logits (its tie-break included), and the logits match the oracle."""
    tdt = TORCH_DT[dt]
    V, K = 32000, 2048
    h = seeded((M, K), 40 + M, 1.0, tdt).to(DEV)
    w = seeded((V, K), 41, 0.02, tdt).to(DEV)
    tok = ob.lm_head_argmax(h, w)
    ob.device_check()
    logits = _gpu_logits(h, w, dt)
    for m in range(M):
        assert int(tok[m]) == orc.argmax_reference(logits[m]), m
    ref = orc.linear(bits(h[:2].cpu()), bits(w.cpu()), dt, "f32")
    assert_close(torch.from_numpy(logits[:2]), torch.from_numpy(ref), "lm head logits",
                 exact_min=EXACT_MIN)


def test_lm_head_argmax_ties():
    """Planted exact ties: identical weight rows give identical logits, and
    the winner follows the reference's order (bit-reversed residue mod 512,
    then position), not simply the first position."""
    V, K, M = 4096, 512, 3
    h = seeded((M, K), 50, 1.0)
    w = seeded((V, K), 51, 0.02)
    top = (seeded((1, K), 52, 1.0).float() * 0.5)[0]
    for m in (0, 2):                                  # the planted rows win on rows 0 and 2
        if float(h[m].float() @ top) < 0:
            h[m] = -h[m]
    h[1] = 0.0                                        # every logit +-0 on row 1: all tie
    for pos in (1, 2, 257, 1026, 3000):               # residues 1, 2, 257, 2, 440
        w[pos] = top.half()
    h, w = h.to(DEV), w.to(DEV)
    tok = ob.lm_head_argmax(h, w)
    ob.device_check()
    logits = _gpu_logits(h, w, 0)
    for m in range(M):
        assert int(tok[m]) == orc.argmax_reference(logits[m]), m
    # 9-bit reversals of the residues: 256, 128, 257, 128, 59 -> position 3000;
    # all-zero logits: residue 0 reverses to 0 -> position 0
    assert [int(t) for t in tok] == [3000, 0, 3000]


def test_reference_entry_points_drop_in():
    """kernels::matmul / fused_silu_mul / add / bf16_to_fp32 / launch_gemm_cute
    with the reference's exact C++ signatures (bf16, default stream)."""
    dt = 1
    tdt = torch.bfloat16
    for M, N, K in ((1, 256, 512), (64, 384, 256), (128, 256, 1024)):
        x = seeded((M, K), 1, 1.0, tdt)
        w = seeded((N, K), 2, 0.02, tdt)
        dx, dw = x.to(DEV), w.to(DEV)  # keep the device copies alive across the calls
        c = torch.empty((M, N), dtype=tdt, device=DEV)
        _lib.shim("kernels::matmul")(c.data_ptr(), dx.data_ptr(), dw.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        ref = orc.linear(bits(x), bits(w), dt, "none")
        assert_close(c.cpu().float(), from_bits(ref, tdt).float(), "kernels::matmul",
                     exact_min=EXACT_MIN)
        c.zero_()
        assert _lib.shim("launch_gemm_cute")(c.data_ptr(), dx.data_ptr(), dw.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        assert_close(c.cpu().float(), from_bits(ref, tdt).float(), "launch_gemm_cute",
                     exact_min=EXACT_MIN)
    n = 5000
    g = seeded((n,), 3, 3.0, tdt)
    u = seeded((n,), 4, 1.0, tdt)
    dg, du = g.to(DEV), u.to(DEV)
    out = torch.empty(n, dtype=tdt, device=DEV)
    _lib.shim("kernels::fused_silu_mul")(out.data_ptr(), dg.data_ptr(), du.data_ptr(), 1, n)
    torch.cuda.synchronize()
    assert (bits(out.cpu()) == orc.silu_mul(bits(g), bits(u), dt)).mean() > 0.999
    xx = g.to(DEV)
    _lib.shim("kernels::add")(xx.data_ptr(), du.data_ptr(), n)
    torch.cuda.synchronize()
    assert np.array_equal(bits(xx.cpu()), orc.add(bits(g), bits(u), dt))
    f = torch.empty(n, dtype=torch.float32, device=DEV)
    _lib.shim("kernels::bf16_to_fp32")(f.data_ptr(), dg.data_ptr(), n)
    torch.cuda.synchronize()
    assert np.array_equal(f.cpu().numpy(), orc.widen(bits(g), dt))


def test_pack_gate_up_matches_oracle():
    IM, K = 704, 2048
    wg = seeded((IM, K), 1, 0.02)
    wu = seeded((IM, K), 2, 0.02)
    wp = ob.pack_gate_up(wg.to(DEV), wu.to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(bits(wp.cpu()), orc.pack_gate_up(bits(wg), bits(wu)))


def test_unfused_path_equals_fused_semantics():
    """gate, up via matmul, then fused_silu_mul == the fused SWIGLU epilogue;
    matmul then add == the RESIDUAL epilogue (same rounding points)."""
    M, IM, K = 96, 256, 512
    x = seeded((M, K), 1, 1.0).to(DEV)
    wg = seeded((IM, K), 2, 0.02).to(DEV)
    wu = seeded((IM, K), 3, 0.02).to(DEV)
    g = ob.linear(x, wg)
    u = ob.linear(x, wu)
    unf = torch.empty_like(g)
    ob.fused_silu_mul(unf, g, u, M, IM)
    fused = ob.linear(x, ob.pack_gate_up(wg, wu), epilogue="swiglu")
    torch.cuda.synchronize()
    assert (unf == fused).float().mean().item() > 0.99
    assert_close(fused.float().cpu(), unf.float().cpu(), "fused vs unfused swiglu")

