"""The CPU oracle against independent references (CPU only).

* a float64 torch restatement of each epilogue with the reference's rounding
  points (kernels/matmul.cu:32-43, kernels/fused_swiglu.cu:11-15,
  kernels/softmax.cu:81,89, src/model.cu:98-130);
* the golden fixtures in tests/golden/, produced by running the reference's
  own kernels (compiled from its sources) on a B200.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import TORCH_DT, assert_close, bits, from_bits, seeded

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def torch_ref(x, w, dt, epi, res=None):
    """float64 accumulation, then the reference's rounding points."""
    tdt = TORCH_DT[dt]
    acc = x.double() @ w.double().T
    r16 = lambda t: t.to(tdt).double()
    if epi == "none":
        return acc.to(tdt)
    if epi == "residual":
        return (res.double() + r16(acc)).to(tdt)
    if epi == "f32":
        return r16(acc).float()
    if epi == "f32_partial":
        return acc.float()
    if epi == "swiglu":
        N = w.shape[0] // 2
        idx = torch.arange(N)
        gr = (idx // 64) * 128 + idx % 64
        g = r16(acc[:, gr]).float()
        u = r16(acc[:, gr + 64]).float()
        return (g / (1.0 + torch.exp(-g)) * u).to(tdt)
    raise ValueError(epi)


@pytest.mark.parametrize("dt", [0, 1])
@pytest.mark.parametrize("epi", ["none", "residual", "f32", "f32_partial", "swiglu"])
@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (5, 192, 200), (33, 128, 1000), (64, 256, 2048)])
def test_oracle_matches_float64(dt, epi, M, N, K):
    tdt = TORCH_DT[dt]
    x = seeded((M, K), 1, 1.0, tdt)
    wrows = 2 * N if epi == "swiglu" else N
    w = seeded((wrows, K), 2, 0.02, tdt)
    res = seeded((M, N), 3, 1.0, tdt) if epi == "residual" else None
    got = orc.linear(bits(x), bits(w), dt, epi, bits(res) if res is not None else None)
    ref = torch_ref(x, w, dt, epi, res)
    if epi in ("f32", "f32_partial"):
        got_t = torch.from_numpy(got)
    else:
        got_t = from_bits(got, tdt)
    assert_close(got_t.float(), ref.float(), f"oracle {epi} dt={dt} {M}x{N}x{K}")


def test_rounding_is_round_to_nearest_even():
    g = torch.Generator().manual_seed(7)
    f = torch.cat([torch.randn(20000, generator=g) * s for s in (1e-6, 1e-3, 1.0, 1e3, 6e4)])
    f = torch.cat([f, torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 65504.0, 65520.0])])
    for dt in (0, 1):
        ours = orc.round16(f.numpy(), dt)
        theirs = bits(f.to(TORCH_DT[dt]))
        assert np.array_equal(ours, theirs)
        back = orc.widen(ours, dt)
        assert np.array_equal(back, f.to(TORCH_DT[dt]).float().numpy())


def test_pack_gate_up_layout():
    IM, K = 192, 16
    wg = np.arange(IM * K, dtype=np.uint16).reshape(IM, K)
    wu = (np.arange(IM * K, dtype=np.uint16) + 30000).reshape(IM, K)
    wp = orc.pack_gate_up(wg, wu)
    for g in range(IM // 64):
        assert np.array_equal(wp[128 * g:128 * g + 64], wg[64 * g:64 * g + 64])
        assert np.array_equal(wp[128 * g + 64:128 * g + 128], wu[64 * g:64 * g + 64])


def test_elementwise_match_torch():
    for dt in (0, 1):
        tdt = TORCH_DT[dt]
        g = seeded((4096,), 11, 3.0, tdt)
        u = seeded((4096,), 12, 1.0, tdt)
        got = from_bits(orc.silu_mul(bits(g), bits(u), dt), tdt)
        gf = g.float()
        ref = (gf / (1.0 + torch.exp(-gf)) * u.float()).to(tdt)
        assert_close(got.float(), ref.float(), "silu_mul")
        got = from_bits(orc.add(bits(g), bits(u), dt), tdt)
        assert torch.equal(got, (g.float() + u.float()).to(tdt))


def test_gemm_f32_baseline_is_exact_enough():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((37, 301), dtype=np.float32)
    W = rng.standard_normal((53, 301), dtype=np.float32)
    C = orc.gemm_f32(A, W)
    np.testing.assert_allclose(C, A.astype(np.float64) @ W.T.astype(np.float64), rtol=1e-4, atol=1e-4)


def _golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: os.path.basename(p))
def test_oracle_matches_reference_golden(path):
    """Outputs of the reference's own kernels (see tests/golden/make_golden.py)."""
    z = np.load(path)
    kind = str(z["kind"])
    dt = 1  # the reference is bf16-only
    path_kind = str(z["path"]) if kind == "matmul" else None
    if kind == "matmul" and path_kind in ("gemv", "rowgemv"):
        # the reference's GEMV (one launch per row in the non-cuBLAS build's
        # fallback): the oracle's restatement of its summation order
        # reproduces the output bit for bit
        rows = [orc.gemv_reference_order(z["A"][m], z["B"], dt) for m in range(int(z["M"]))]
        assert np.array_equal(np.concatenate(rows), z["C"])
        K = int(z["K"])
        T = min(K, 256)
        if T & (T - 1) == 0:
            # power-of-two block: nothing dropped, the plain oracle agrees too
            full = orc.linear(z["A"], z["B"], dt, "none")
            assert (full == z["C"]).mean() >= 0.97
    elif kind == "matmul":
        got = orc.linear(z["A"], z["B"], dt, "none")
        ref = z["C"]
        # same arithmetic up to fp32 summation order: nearly all bit-identical
        assert (got == ref).mean() >= 0.97
        assert_close(from_bits(got, torch.bfloat16).float(), from_bits(ref, torch.bfloat16).float(),
                     f"golden {os.path.basename(path)}")
    elif kind == "silu_mul":
        got = orc.silu_mul(z["gate"], z["up"], dt)
        # expf on the GPU and in libm may differ in the last fp32 ulp, which
        # can flip a bf16 rounding now and then
        assert (got == z["out"]).mean() >= 0.999
    elif kind == "add":
        got = orc.add(z["x"], z["y"], dt)
        assert np.array_equal(got, z["out"])
    elif kind == "bf16_to_fp32":
        assert np.array_equal(orc.widen(z["x"], dt), z["out"])
    else:
        pytest.fail(f"unknown golden kind {kind}")


def test_golden_fixtures_present():
    files = _golden_files()
    kinds = {str(np.load(p)["kind"]) for p in files}
    assert {"matmul", "silu_mul", "add", "bf16_to_fp32"} <= kinds, (
        "tests/golden is missing reference fixtures; regenerate with "
        "tests/golden/make_golden.py on a GPU")


def test_argmax_key_order_matches_the_reference_sampler():
    """The fused LM-head argmax packs the reference sampler's choice into an
    order (value, bit-reversed residue mod 512, position); check that order
    against the literal restatement of the 512-thread kernel on tie-heavy rows
    (few distinct values, -inf, NaN, nothing valid)."""
    rng = np.random.default_rng(5)
    for trial in range(200):
        n = int(rng.integers(1, 2600))
        x = rng.integers(-3, 4, size=n).astype(np.float32)
        if trial % 5 == 0:
            x[rng.integers(0, n, size=n // 3)] = -np.inf
        if trial % 9 == 0:
            x[rng.integers(0, n, size=n // 4)] = np.nan
        if trial % 17 == 0:
            x[:] = -np.inf
        assert orc.argmax_reference(x) == orc.argmax_key_order(x), trial


def _elf_dynamic_flags(path):
    """(DT_FLAGS value, DT_SYMBOLIC present) from an ELF64 little-endian file."""
    import struct
    data = open(path, "rb").read()
    assert data[:4] == b"\x7fELF" and data[4] == 2 and data[5] == 1
    e_phoff, = struct.unpack_from("<Q", data, 0x20)
    e_phentsize, e_phnum = struct.unpack_from("<HH", data, 0x36)
    flags, symbolic = 0, False
    for i in range(e_phnum):
        p_type, _, p_offset, _, _, p_filesz = struct.unpack_from("<IIQQQQ", data,
                                                                 e_phoff + i * e_phentsize)
        if p_type != 2:  # PT_DYNAMIC
            continue
        for j in range(p_filesz // 16):
            tag, val = struct.unpack_from("<qQ", data, p_offset + 16 * j)
            if tag == 0:
                break
            if tag == 30:  # DT_FLAGS
                flags = val
            if tag == 16:  # DT_SYMBOLIC
                symbolic = True
    return flags, symbolic


@pytest.mark.parametrize("path", [orc.REF_CUBLAS, orc.REF_CUTE])
def test_reference_checkers_bind_their_own_kernels(path):
    """The checkers built from the reference's sources define the same
    kernels:: names as liborin_b200.so's drop-in entry points; linked with
    -Bsymbolic, their entry points reach the reference's kernels even in a
    process that also loaded liborin_b200.so."""
    if not path.exists():
        pytest.skip(f"{path.name} not built")
    flags, symbolic = _elf_dynamic_flags(path)
    assert symbolic or (flags & 0x2), f"{path.name} is not linked -Bsymbolic"


def test_library_symbols_stay_out_of_the_global_scope():
    import ctypes
    from orininfer_b200 import _lib
    assert hasattr(_lib.lib, "orin_linear")
    assert not hasattr(ctypes.CDLL(None), "orin_linear")


def test_reference_cute_kernel_is_not_launchable():
    """The reference's CuTe kernel (gemm_multi_stage) made an illegal address
    access on a B200, so nothing here may launch it: the checker library exports
    no entry for it, and the build without cuBLAS refuses every shape that
    kernels::matmul would send to it (tile-aligned M, N, K), both in Python and
    in the C entry point, before any CUDA call.  Unaligned shapes keep the
    per-row GEMV fallback that the rowgemv fixture pins."""
    import ctypes
    assert orc.cute_refused(128, 256, 512)
    assert orc.cute_refused(4096, 4096, 4096)
    assert not orc.cute_refused(3, 64, 96)      # the rowgemv fixture's shape
    assert not orc.cute_refused(1, 128, 128)    # M == 1 is the GEMV
    assert not orc.cute_refused(128, 100, 64)
    if not orc.REF_CUTE.exists():
        pytest.skip("libref_cute.so not built")
    raw = ctypes.CDLL(str(orc.REF_CUTE), mode=os.RTLD_LOCAL | os.RTLD_NOW)
    assert not hasattr(raw, "ref_gemm_cute")
    raw.ref_matmul.restype = ctypes.c_int
    raw.ref_matmul.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    # null pointers: the refusal returns before anything touches them or the GPU
    assert raw.ref_matmul(None, None, None, 128, 256, 512) == orc.REF_REFUSED_CUTE
    rk = orc.RefKernels(cute=True)
    assert not hasattr(rk, "gemm_cute")
    with pytest.raises(ValueError, match="CuTe"):
        rk.matmul(0, 0, 0, 256, 128, 64)
