"""Failure detection on the device without a GPU fault.

Every mbarrier wait in this library's kernels is bounded: past its limit it
records a timeout in the context's status word and the kernel unwinds, so a
lost arrival surfaces as ESMCU_ERR_TIMEOUT instead of a hung GPU.  Here a
small kernel waits, through the same bounded-wait helpers, on an mbarrier
that is given one of its two expected arrivals, with a short limit; the test
checks that the host gets the status, that every waiter gave up, and that the
context then serves normal calls.  Nothing faults, traps or hangs: each wait
ends by itself after the limit.
"""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(cuda):
    """The context the kernel-facade ops use on device 0, so the normal calls
    after a timeout run on the very context that reported it."""
    from esm_b200 import ops

    return ops.context(0)


def _selftest(ctx, limit_us):
    from esm_b200 import _lib

    n = C.c_int(-1)
    t0 = time.perf_counter()
    rc = _lib.lib().esmcu_bounded_wait_selftest(ctx, limit_us, C.byref(n))
    return rc, n.value, time.perf_counter() - t0


def test_bounded_wait_runs_out_and_reports_timeout(ctx):
    from esm_b200 import _lib

    rc, released, secs = _selftest(ctx, 20_000)
    assert _lib.STATUS[rc] == "TIMEOUT", _lib.lib().esmcu_last_error()
    assert b"bound" in _lib.lib().esmcu_last_error()
    assert released == 4  # the plain waiter and the three abort-flag waiters
    assert 0.02 <= secs < 2.0, secs


def test_context_serves_normal_calls_after_a_timeout(ctx, cuda, O):
    import torch

    from esm_b200 import _lib, ops

    rc, _, _ = _selftest(ctx, 5_000)
    assert _lib.STATUS[rc] == "TIMEOUT"
    # The status word was cleared when it was read: the context is clean.
    _lib.call("esmcu_synchronize", ctx)
    # A normal op on the same device still gives the oracle's bits.
    rng = np.random.default_rng(3)
    A = rng.standard_normal((96, 256)).astype(np.float32)
    Wq, ws = O.quantize_weights((rng.standard_normal((64, 256)) * 0.02).astype(np.float32))
    C_ = ops.linear_int8(torch.from_numpy(A).to(cuda), torch.from_numpy(Wq).to(cuda),
                         torch.from_numpy(ws).to(cuda))
    ops.synchronize()
    assert np.array_equal(C_.cpu().numpy(), O.linear_int8(A, Wq, ws))
    # And the self-test is repeatable.
    rc, released, _ = _selftest(ctx, 5_000)
    assert _lib.STATUS[rc] == "TIMEOUT" and released == 4
    _lib.call("esmcu_synchronize", ctx)


def test_selftest_rejects_bad_limits(ctx):
    from esm_b200 import _lib

    for bad in (0, -5, 2_000_000):
        rc, _, _ = _selftest(ctx, bad)
        assert _lib.STATUS[rc] == "INVALID_ARGUMENT"
