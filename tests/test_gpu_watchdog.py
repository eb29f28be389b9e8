"""The device-side watchdog, exercised without any fault: a bounded wait is
made to run out (its flag is never set) and the host reads the status."""
import time

import pytest
import torch

import orininfer_b200 as ob
from orininfer_b200 import _lib
from oracle import oracle as orc
from tests._util import EXACT_MIN, assert_close, bits, from_bits, seeded

pytestmark = pytest.mark.gpu


def test_peer_wait_gives_up_and_the_context_stays_usable():
    ob.device_check()                      # nothing pending before
    s = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    assert _lib.lib.orin_p2p_watchdog_selftest(s) == _lib.OK
    waited = time.time() - t0
    assert 1.5 < waited < 60, waited       # the 2 s bound, not a hang
    assert _lib.lib.orin_device_check(s) == _lib.ERR_TIMEOUT
    assert _lib.lib.orin_device_check(s) == _lib.OK   # the record was cleared
    # the same context still computes correctly
    x = seeded((4, 256), 1, 1.0)
    w = seeded((128, 256), 2, 0.02)
    y = ob.linear(x.cuda(), w.cuda())
    ob.device_check()
    ref = orc.linear(bits(x), bits(w), 0)
    assert_close(y.cpu().float(), from_bits(ref, torch.float16).float(), "after the watchdog",
                 exact_min=EXACT_MIN)
