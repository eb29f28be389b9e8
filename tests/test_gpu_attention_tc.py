"""The two attention kernels forced one at a time, against the oracle (B200
only): the tcgen05 prefill kernel (csrc/attention_tc.cu: S and P.V on the
tensor cores, accumulators in tensor memory) with one query tile per CTA
("tc1") and, for head dim 64, two paired tiles ("tc2"; head dim 128 runs the
one-tile form there too), and the mma.sync kernel
(csrc/attention.cu) on every shape the tcgen05 kernel takes — prefill chunks
that fill and wrap the ring, small windows wrapped many times, MHA, GQA groups
of 4, 8, 64 and 128 heads, head dims 64 and 128, rows left over in the last
block.

The kernel is forced with the ORIN_ATTN_KERNEL tuning override, which the
library reads once per process, so each kernel runs in its own subprocess.
Tolerance: the attention bar of the other attention tests (max relative error
1e-2 of the largest output, mean absolute error 1e-3)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

TINY = dict(nh=32, nkv=4, hd=64)
LLAMA3 = dict(nh=32, nkv=8, hd=128)
CASES = [
    # (S, C, shape, n_sink, W)
    (16, 16, TINY, 4, 1024),        # one row block, one key tile
    (1028, 1028, TINY, 4, 1024),    # first chunk: sinks + a full window
    (1020, 2048, TINY, 4, 1024),    # second chunk: wraps the ring onto itself
    (130, 2000, TINY, 4, 1024),     # a short chunk deep into the sequence
    (300, 300, LLAMA3, 4, 1024),    # head dim 128
    (500, 1300, LLAMA3, 4, 1024),   # head dim 128, wrapped
    (77, 600, dict(nh=8, nkv=2, hd=64), 4, 80),      # many ring wraps, small window
    (200, 200, dict(nh=16, nkv=16, hd=128), 0, 16),  # MHA, no sink, tiny window
    (5, 1000, dict(nh=64, nkv=1, hd=64), 4, 200),    # group of 64
    (3, 50, dict(nh=128, nkv=1, hd=64), 4, 32),      # group of 128
    (2, 300, dict(nh=256, nkv=1, hd=64), 4, 256),    # group of 256: two row blocks per token
]


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["tc1", "tc2", "mma"])
def test_forced_attention_kernel_matches_oracle(kernel):
    env = dict(os.environ, ORIN_ATTN_KERNEL=kernel, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, os.path.abspath(__file__)], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"kernel {kernel}:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"


def _main() -> None:
    import numpy as np
    import torch

    from oracle import oracle as O
    from orininfer_b200 import kernels as K
    from tests._util import TORCH_DT, assert_close, from_bits

    def rand16(rng, shape, dt):
        return O.round16(rng.standard_normal(shape).astype(np.float32), dt)

    def dev(a, dt):
        return from_bits(a, TORCH_DT[dt]).cuda()

    K.device_check()  # sets the device up, so every kernel below records a timeout
    for dt in (0, 1):
        for i, (S, C, shape, ns, W) in enumerate(CASES):
            nh, nkv, hd = shape["nh"], shape["nkv"], shape["hd"]
            rng = np.random.default_rng(100 * i + dt)
            q = rand16(rng, (S, nh, hd), dt)
            kp = rand16(rng, (ns + W, nkv, hd), dt)
            vp = rand16(rng, (ns + W, nkv, hd), dt)
            scale = hd ** -0.5
            r = O.attention(q, kp, vp, S, C, nh, nkv, hd, scale, ns, W, dt)
            out = torch.empty((S, nh, hd), dtype=TORCH_DT[dt], device="cuda")
            K.attention(out, dev(q, dt), dev(kp, dt), dev(vp, dt), S, C, nh, nkv, hd, scale, ns,
                        W)
            K.device_check()
            what = (f"{os.environ.get('ORIN_ATTN_KERNEL')} dt={dt} S={S} C={C} {shape} "
                    f"n_sink={ns} W={W}")
            assert_close(out.cpu().float(), from_bits(r, TORCH_DT[dt]).float(), what)
            print("passed", what, flush=True)

    # slots that no call has written yet hold NaN bits: a first chunk that
    # fills part of the ring must not read them
    dt, S, ns, W = 1, 600, 4, 1024
    nh, nkv, hd = TINY["nh"], TINY["nkv"], TINY["hd"]
    rng = np.random.default_rng(7)
    q = rand16(rng, (S, nh, hd), dt)
    kp = rand16(rng, (ns + W, nkv, hd), dt)
    vp = rand16(rng, (ns + W, nkv, hd), dt)
    kp[S:] = 0x7FC0
    vp[S:] = 0x7FC0
    r = O.attention(q, kp, vp, S, S, nh, nkv, hd, hd ** -0.5, ns, W, dt)
    out = torch.empty((S, nh, hd), dtype=TORCH_DT[dt], device="cuda")
    K.attention(out, dev(q, dt), dev(kp, dt), dev(vp, dt), S, S, nh, nkv, hd, hd ** -0.5, ns, W)
    K.device_check()
    assert not torch.isnan(out.float()).any()
    assert_close(out.cpu().float(), from_bits(r, TORCH_DT[dt]).float(), "unwritten NaN slots")
    print("ok")


if __name__ == "__main__":
    _main()
