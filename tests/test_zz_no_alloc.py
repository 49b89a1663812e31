"""esmcu_linear_int8_noalloc: the W8A8 Linear for callers that cannot let the
library allocate device memory (a process that has handed its HBM to its own
pool, or that cannot take an allocation's synchronisation mid-stream).  Its
scratch is a fixed array built into the library and shared by every call on a
device, so each case makes two calls in a row -- the first with larger
activations than the second, so a stale absmax left by the first would change
the second's result -- and compares both, through the C-ABI alone, with the
allocating esmcu_linear_int8 on the same inputs and with the CPU oracle
(quantise, exact int32 dot, FinalizeStore16 dequant).  All three agree bit for
bit, the tolerance of the INT8 GEMM tests.  The device's free memory is also
read around repeated calls: a call that allocated would lower it.

This file is collected last on purpose; it also passes when run on its own.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


@pytest.fixture(scope="module")
def ctx():
    from esm_b200 import _lib

    n = C.c_int(0)
    if _lib.lib().esmcu_device_count(C.byref(n)) != 0 or n.value == 0:
        pytest.skip("no CUDA device")
    h = C.c_void_p()
    _lib.call("esmcu_open", 0, C.byref(h))
    yield h
    _lib.call("esmcu_close", h)


class _Dev:
    """Device buffers owned by the test (esmcu_malloc), freed on exit."""

    def __init__(self, ctx):
        self.ctx, self.ptrs = ctx, []

    def put(self, a):
        from esm_b200 import _lib

        p = C.c_void_p()
        _lib.call("esmcu_malloc", self.ctx, max(a.nbytes, 1), C.byref(p))
        self.ptrs.append(p)
        _lib.call("esmcu_memcpy_h2d", self.ctx, p, a.ctypes.data, a.nbytes)
        return p

    def get(self, p, shape, dtype):
        from esm_b200 import _lib

        out = np.empty(shape, dtype)
        _lib.call("esmcu_synchronize", self.ctx)
        _lib.call("esmcu_memcpy_d2h", self.ctx, out.ctypes.data, p, out.nbytes)
        return out

    def free(self):
        from esm_b200 import _lib

        for p in self.ptrs:
            _lib.call("esmcu_free", self.ctx, p)


def _weights(rng, N, K):
    Wq = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = (rng.random(N, dtype=np.float32) * 0.02 + 1e-3).astype(np.float32)
    return Wq, ws


def _free_bytes():
    import torch

    torch.cuda.synchronize()
    return torch.cuda.mem_get_info(0)[0]


@pytest.mark.parametrize("act_quant", [0, 1])
@pytest.mark.parametrize("M,N,K,w_offset", [(512, 1280, 1280, 0), (300, 257, 1000, 0),
                                             (7, 33, 23, 0), (64, 96, 1280, 3)])
def test_two_calls_match_allocating_entry_point(ctx, M, N, K, w_offset, act_quant):
    """w_offset > 0 passes W at an address that is not 16-byte aligned (with
    K % 16 == 0), which takes the padded-copy path."""
    import oracle as O

    from esm_b200 import _lib

    rng = np.random.default_rng(M * 7 + N * 3 + K + act_quant)
    Wq, ws = _weights(rng, N, K)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    d = _Dev(ctx)
    try:
        W_store = np.zeros(N * K + 16, np.int8)
        W_store[w_offset:w_offset + N * K] = Wq.ravel()
        dW = C.c_void_p(d.put(W_store).value + w_offset)
        dws, db = d.put(ws), d.put(bias)
        dC_ref = d.put(np.zeros((M, N), np.float32))
        dC = d.put(np.zeros((M, N), np.float32))
        for call, amp in enumerate((10.0, 1.0)):
            A = (rng.standard_normal((M, K)) * amp).astype(np.float32)
            dA = d.put(A)
            _lib.call("esmcu_linear_int8", ctx, dA, dW, dws, db, dC_ref, M, N, K, act_quant)
            want = d.get(dC_ref, (M, N), np.float32)
            _lib.call("esmcu_linear_int8_noalloc", ctx, dA, dW, dws, db, dC, M, N, K, act_quant)
            got = d.get(dC, (M, N), np.float32)
            assert np.isfinite(got).all()
            assert np.array_equal(got, want), (
                f"call {call}: max |diff| {np.abs(got - want).max():.3e}")
            oracle = O.linear_int8(A, Wq, ws, bias, per_token=act_quant == 1)
            assert np.array_equal(got, oracle), (
                f"call {call}: vs oracle max |diff| {np.abs(got - oracle).max():.3e}")
    finally:
        d.free()


def test_calls_allocate_no_device_memory(ctx):
    from esm_b200 import _lib

    M, N, K = 2048, 1280, 1280
    rng = np.random.default_rng(11)
    Wq, ws = _weights(rng, N, K)
    d = _Dev(ctx)
    try:
        dA = d.put(rng.standard_normal((M, K)).astype(np.float32))
        dW, dws = d.put(Wq), d.put(ws)
        dC = d.put(np.zeros((M, N), np.float32))
        before = _free_bytes()
        for _ in range(3):
            _lib.call("esmcu_linear_int8_noalloc", ctx, dA, dW, dws, None, dC, M, N, K, 0)
        _lib.call("esmcu_synchronize", ctx)
        assert _free_bytes() == before
    finally:
        d.free()


def test_rejects_shapes_beyond_the_fixed_scratch(ctx):
    from esm_b200 import EsmCudaError, _lib

    M, N, K = 16384, 64, 1280  # 16384 * 1280 int8 codes alone exceed 16 MiB
    assert M * K > SCRATCH_BYTES
    d = _Dev(ctx)
    try:
        dA = d.put(np.zeros((M, K), np.float32))
        dW, dws = d.put(np.zeros((N, K), np.int8)), d.put(np.ones(N, np.float32))
        dC = d.put(np.zeros((M, N), np.float32))
        with pytest.raises(EsmCudaError, match="fixed scratch holds") as ei:
            _lib.call("esmcu_linear_int8_noalloc", ctx, dA, dW, dws, None, dC, M, N, K, 0)
        assert _lib.STATUS[ei.value.code] == "OUT_OF_RANGE"
        # The context stays usable after the rejection.
        _lib.call("esmcu_linear_int8_noalloc", ctx, dA, dW, dws, None, dC, 64, N, K, 0)
        _lib.call("esmcu_synchronize", ctx)
    finally:
        d.free()
