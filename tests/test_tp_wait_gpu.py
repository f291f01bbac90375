"""The bounded cross-rank wait of the fused peer-store tensor-parallel
reduction runs out cleanly, on one GPU and without a second rank: the real
detail::tp_p2p_residual_kernel is launched (through the test-only hook
tests/native/libtp_wait_hook.so) for a world of two whose second rank never
arrives, with a 200 ms limit. The kernel must

* return after the limit (not hang), leave the context usable, and report
  error 6 in the per-device error word the engine reads after every step;
* leave the arrival counter as the ranks left it (a slow rank's late tiles
  must not land in a re-armed counter) and the hidden rows untouched;

and with every arrival in place it must sum the slots in rank order, add
them to the hidden rows and re-arm the counter. The wait ends by itself;
nothing waits on another kernel.
"""

import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

HOOK = os.path.join(os.path.dirname(os.path.abspath(__file__)), "native", "libtp_wait_hook.so")


def test_peer_wait_runs_out_and_reports_error_6():
    if not os.path.exists(HOOK):
        pytest.fail("tests/native/libtp_wait_hook.so is missing: run __graft_entry__.build()")
    torch.cuda.init()
    lib = ctypes.CDLL(HOOK)
    lib.opw_test_tp_wait.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
    lib.opw_test_tp_wait.restype = ctypes.c_int
    out = np.zeros(8, np.float64)
    assert lib.opw_test_tp_wait(200, out.ctypes.data_as(ctypes.POINTER(ctypes.c_double))) == 0
    err, cnt, ms, moved, err_ok, cnt_ok, sum_err = out[:7]
    assert err == 6, out
    assert cnt == 5, out  # not re-armed after the wait ran out
    assert moved == 0.0, out
    assert 150.0 <= ms <= 5000.0, out
    assert err_ok == 0 and cnt_ok == 0, out
    assert sum_err <= 1e-6, out
    # the context is still usable
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().cpu()) == 8.0
