"""Failure handling on one GPU, without a fault: a bounded device wait that runs out.

The one-shot allreduce's peer wait is exercised by n730_tp_wait_check as rank 0 of
2 with a local stand-in for rank 1's exchange region that nothing writes: every
slice's wait ends after a short limit (5 ms), the kernel sets the device error word
and returns, and the host reads N730_TIMEOUT (-15).  The context stays usable:
the same op with the peer's slice present completes with the right sum, and an
ordinary GEMV runs after it.
"""
import ctypes as C
import time

import numpy as np
import pytest

from n730_b200 import _lib

pytestmark = pytest.mark.gpu


def test_peer_wait_runs_out_and_context_survives():
    import torch
    lib = _lib.cuda()
    torch.cuda.set_device(0)
    t0 = time.monotonic()
    assert lib.n730_tp_wait_check(5_000_000, 0, None) == -15
    assert time.monotonic() - t0 < 2.0
    assert lib.n730_tp_wait_check(5_000_000, 1, None) == 0  # a clean op right after
    # ordinary work still runs: a small GEMV through the C ABI
    rows, cols = 64, 128
    codes = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda")
    s16 = torch.full((rows, 1), 0.01, dtype=torch.float16, device="cuda")
    z16 = torch.full((rows, 1), 8.0, dtype=torch.float16, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    q = C.c_void_p()
    _lib.check(lib.n730_qweight_create(0x44, rows, cols, 128, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                       C.byref(q)), "create")
    x = torch.ones(1, cols, device="cuda")
    y = torch.empty(1, rows, device="cuda")
    _lib.check(lib.n730_qlinear(q, P(x), cols, 1, P(y), rows, None, None, 0, None, 1e-6, 0, None), "qlinear")
    torch.cuda.synchronize()
    lib.n730_qweight_destroy(q)
    assert np.isfinite(y.cpu().numpy()).all()


def test_wait_check_rejects_bad_limits():
    lib = _lib.cuda()
    assert lib.n730_tp_wait_check(0, 0, None) == -13
    assert lib.n730_tp_wait_check(20_000_000_000, 0, None) == -13
