"""orin_tp_linear_row_static: the row-parallel linear with its partial sums in
a file-scope device array instead of a caller buffer.

On the GPU (one rank, NCCL communicator of size 1): two consecutive calls of
different shapes must give exactly the bits of orin_tp_linear_row with a
caller buffer (same kernels, same summation order), and match the oracle.
Without a GPU: argument checks that return before any device work."""
import ctypes

import pytest
import torch

from orininfer_b200 import _lib


def _call_static(comm, out, x, w, M, N, K, dt, res, stream=None):
    s = torch.cuda.current_stream() if stream is None else stream
    return _lib.lib.orin_tp_linear_row_static(
        comm, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(w.data_ptr()), M, N, K, dt,
        ctypes.c_void_p(res.data_ptr()) if res is not None else None,
        ctypes.c_void_p(s.cuda_stream))


def test_static_partial_capacity_and_argument_checks():
    cap = _lib.lib.orin_tp_static_partial_capacity()
    assert cap == 16 << 20
    dummy = ctypes.c_void_p(16)
    # null communicator / operands and non-positive sizes: rejected on the host
    assert _lib.lib.orin_tp_linear_row_static(None, dummy, dummy, dummy, 4, 4, 8, 0, None,
                                              None) == _lib.ERR_INVALID_ARG
    assert _lib.lib.orin_tp_linear_row_static(dummy, dummy, dummy, dummy, 0, 4, 8, 0, None,
                                              None) == _lib.ERR_INVALID_ARG


@pytest.mark.gpu
def test_static_scratch_matches_caller_scratch_on_two_calls():
    import orininfer_b200 as ob
    from oracle import oracle as orc
    from orininfer_b200 import tp
    from tests._util import EXACT_MIN, assert_close, bits, from_bits, seeded

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    comm = tp.TPComm(0, 1, 0, tp.TPComm.unique_id(), timeout_s=30.0)
    try:
        for call, (M, N, K, dt) in enumerate(((96, 1024, 2048, 0), (33, 768, 512, 1))):
            tdt = torch.float16 if dt == 0 else torch.bfloat16
            x = seeded((M, K), 10 + call, 1.0, tdt)
            w = seeded((N, K), 20 + call, 0.02, tdt)
            res = seeded((M, N), 30 + call, 1.0, tdt)
            dx, dw, dr = x.to(dev), w.to(dev), res.to(dev)
            ref_out = comm.linear_row(dx, dw, residual=dr)            # caller scratch
            out = torch.empty((M, N), dtype=tdt, device=dev)
            assert _call_static(comm._h, out, dx, dw, M, N, K, dt, dr) == _lib.OK, \
                _lib.lib.orin_last_error()
            comm.wait()
            ob.device_check()
            assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), f"call {call}"
            oracle = orc.linear(bits(x), bits(w), dt, "residual", bits(res))
            assert_close(out.cpu().float(), from_bits(oracle, tdt).float(),
                         f"static scratch call {call}", exact_min=EXACT_MIN)
        # more partial sums than the array holds: rejected before any device work
        big = 1 << 13
        dummy = torch.empty(8, dtype=torch.float16, device=dev)
        assert _call_static(comm._h, dummy, dummy, dummy, big, big * 2 + 8, 64, 0,
                            None) == _lib.ERR_UNSUPPORTED
    finally:
        torch.cuda.synchronize()
        comm.close()


_CAPTURE_PROBE = r"""
import ctypes, sys, torch
sys.path.insert(0, sys.argv[1])
from orininfer_b200 import _lib, tp
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
comm = tp.TPComm(0, 1, 0, tp.TPComm.unique_id(), timeout_s=30.0)
M, N, K = 16, 256, 128
x = torch.randn(M, K, device=dev).half()
w = (torch.randn(N, K, device=dev) * 0.02).half()
out = torch.empty(M, N, device=dev, dtype=torch.float16)
args = lambda s: (comm._h, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                  ctypes.c_void_p(w.data_ptr()), M, N, K, 0, None, ctypes.c_void_p(s.cuda_stream))
s = torch.cuda.Stream()
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=s):
    st = _lib.lib.orin_tp_linear_row_static(*args(s))
msg = _lib.lib.orin_last_error()
assert st == _lib.ERR_INVALID_ARG, (st, msg)
assert b"stream-captured" in (msg if isinstance(msg, bytes) else str(msg).encode()), msg
# outside capture the look-up succeeds and the call computes
with torch.cuda.stream(s):
    st = _lib.lib.orin_tp_linear_row_static(*args(s))
assert st == _lib.OK, _lib.lib.orin_last_error()
comm.wait()
ref = torch.nn.functional.linear(x.float(), w.float())
assert (out.float() - ref).abs().max().item() < 2e-2
torch.cuda.synchronize()
del g
comm.close()
print("CAPTURE_PROBE_OK")
"""


@pytest.mark.gpu
def test_first_static_call_under_capture_is_refused():
    """The first call on a device looks the array's address up, which may load
    the module; made inside stream capture it would break the capture, so it is
    refused with ORIN_ERR_INVALID_ARG and a message, and the next uncaptured
    call works.  Runs in a fresh process, where no earlier call did the
    look-up."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _CAPTURE_PROBE, root], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "CAPTURE_PROBE_OK" in r.stdout, r.stdout + r.stderr
