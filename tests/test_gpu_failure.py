"""The device timeout path on the GPU, made to run out on purpose: a bounded mbarrier wait on a phase that nothing
completes (no trap, no fault, no unbounded loop) must set its status bit, be read back through spanqr_read_status,
and leave the context usable for the next orth call."""
import ctypes

import pytest
import torch

from spanqr_b200 import _lib, orth
from tests import cases

pytestmark = pytest.mark.gpu
DEVICE_FAILURE = 5   # SPANQR_ERR_DEVICE
SELFTEST_BIT = 0x80


def test_wait_that_runs_out_sets_status_and_context_stays_usable():
    L = _lib.lib()
    X = cases.cfg3_matrix(0, K=1024).cuda()
    before = orth(X)
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    s = ctypes.c_int(-1)
    _lib.check(L.spanqr_selftest_timeout(ws.data_ptr(), ws.numel(), 1_000_000, 1, st), "selftest (arrived)")
    assert L.spanqr_read_status(ws.data_ptr(), st, ctypes.byref(s)) == 0 and s.value == 0
    _lib.check(L.spanqr_selftest_timeout(ws.data_ptr(), ws.numel(), 1_000_000, 0, st), "selftest (never arrived)")
    assert L.spanqr_read_status(ws.data_ptr(), st, ctypes.byref(s)) == DEVICE_FAILURE
    assert s.value & SELFTEST_BIT
    after = orth(X)
    torch.cuda.synchronize()
    assert torch.equal(before.view(torch.int32), after.view(torch.int32))
