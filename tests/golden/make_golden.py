"""Regenerate tests/golden/*.npz from the reference's own kernels.

Run on a machine with an sm_100 GPU, after `make -C oracle ref` built
oracle/_ref/ from the reference sources:

    python tests/golden/make_golden.py [outdir]

Each fixture holds seeded bf16 inputs (as uint16 bit patterns) and the
reference kernel's output for them:
  matmul      kernels::matmul — M==1 runs gemv_kernel (kernels/matmul.cu:25-44),
              M>1 runs cublasGemmEx (kernels/matmul.cu:59-68); the "rowgemv"
              fixture is the non-cuBLAS build with an unaligned M, which takes
              the per-row GEMV fallback (kernels/matmul.cu:71-77) without
              launching the CuTe kernel (its alignment check, gemm_cute.cu:302,
              returns first).  The CuTe kernel itself is not run: built for
              sm_100a it raised an illegal-address error on a B200 (its
              128-thread copy layouts under a 256-thread MMA index past the
              tile).
  silu_mul    kernels::fused_silu_mul (kernels/fused_swiglu.cu)
  add         kernels::add (kernels/softmax.cu:78-83)
  bf16_to_fp32 kernels::bf16_to_fp32 (kernels/softmax.cu:87-90)
Inputs: x ~ N(0,1), W ~ N(0, 0.02^2), drawn in fp32 from torch.manual_seed
and cast to bf16.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import RefKernels  # noqa: E402


def seeded(shape, seed, scale):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)


def u16(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def main(out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    dev = torch.device("cuda:0")
    ref = RefKernels(cute=False)
    cute = RefKernels(cute=True)
    seed = 100
    # (name, M, N, K, which library, which reference code path runs)
    cases = [
        ("gemv_1x256x512", 1, 256, 512, ref, "gemv"),
        ("gemv_1x2048x2048", 1, 2048, 2048, ref, "gemv"),
        ("gemv_1x96x200", 1, 96, 200, ref, "gemv"),
        ("cublas_16x384x256", 16, 384, 256, ref, "cublas"),
        ("cublas_128x256x1024", 128, 256, 1024, ref, "cublas"),
        ("cublas_33x100x72", 33, 100, 72, ref, "cublas"),
        ("rowgemv_3x64x96", 3, 64, 96, cute, "rowgemv"),
    ]
    for name, M, N, K, lib, path in cases:
        seed += 1
        A = seeded((M, K), seed, 1.0)
        B = seeded((N, K), seed + 1000, 0.02)
        dA, dB = A.to(dev), B.to(dev)
        dC = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        lib.matmul(dC.data_ptr(), dA.data_ptr(), dB.data_ptr(), M, N, K)
        lib.sync()
        np.savez_compressed(os.path.join(out_dir, f"matmul_{name}.npz"), kind="matmul", path=path,
                            A=u16(A), B=u16(B), C=u16(dC), M=M, N=N, K=K)
        print("wrote", name, flush=True)
    # every device buffer is held in a variable for as long as a kernel uses it
    n = 3 * 4096 + 17
    g = seeded((n,), 501, 3.0)
    u = seeded((n,), 502, 1.0)
    dg, du = g.to(dev), u.to(dev)
    dout = torch.empty(n, dtype=torch.bfloat16, device=dev)
    ref.fused_silu_mul(dout.data_ptr(), dg.data_ptr(), du.data_ptr(), 1, n)
    ref.sync()
    np.savez_compressed(os.path.join(out_dir, "silu_mul.npz"), kind="silu_mul", gate=u16(g),
                        up=u16(u), out=u16(dout))
    x = seeded((n,), 503, 1.0)
    y = seeded((n,), 504, 1.0)
    dx, dy = x.to(dev), y.to(dev)
    ref.add(dx.data_ptr(), dy.data_ptr(), n)
    ref.sync()
    np.savez_compressed(os.path.join(out_dir, "add.npz"), kind="add", x=u16(x), y=u16(y),
                        out=u16(dx))
    dx2 = x.to(dev)
    df = torch.empty(n, dtype=torch.float32, device=dev)
    ref.bf16_to_fp32(df.data_ptr(), dx2.data_ptr(), n)
    ref.sync()
    np.savez_compressed(os.path.join(out_dir, "bf16_to_fp32.npz"), kind="bf16_to_fp32",
                        x=u16(x), out=df.cpu().numpy())
    print("done", flush=True)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
