"""The activation quantisers (quant_bits in csrc/common.cuh) round without a
float-to-int conversion: v = clamp(x * inv, -127, 127), then v + 1.5 * 2^23
in the float adder rounds v to the nearest integer, ties to even, and the low
byte of the sum's bit pattern is q.  This pins that identity in IEEE float32
arithmetic (numpy) against the reference's rule q = clamp(rne(x * inv), +-127)
(gemm_int8.cpp:391-508, pack.cpp:119-132) on ties, bounds and random values."""
import numpy as np

F32 = np.float32


def _adder_q(x, inv):
    # fmax / fmin: like the device's fmaxf / fminf, a NaN operand yields the
    # other one (np.clip would propagate the NaN).
    v = np.fmin(np.fmax((x * inv).astype(F32), F32(-127.0)), F32(127.0)).astype(F32)
    bits = (v + F32(12582912.0)).astype(F32).view(np.uint32)
    return (bits & np.uint32(0xFF)).astype(np.uint8).view(np.int8)


def _reference_q(x, inv):
    return np.clip(np.rint((x * inv).astype(F32)), -127, 127).astype(np.int8)


def test_ties_and_bounds():
    x = np.concatenate([np.arange(-130, 130, dtype=F32) + F32(0.5), np.arange(-130, 131, dtype=F32),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 126.49999, 126.5, 126.50001, -127.5, 127.5,
                                  1e9, -1e9, np.inf, -np.inf], F32)])
    inv = F32(1.0)
    assert np.array_equal(_adder_q(x, inv), _reference_q(x, inv))


def test_random_scales_and_values():
    rng = np.random.default_rng(0)
    for _ in range(20):
        amax = F32(abs(rng.standard_normal()) * 10 ** rng.uniform(-3, 3))
        s = F32(amax / F32(127.0))
        inv = F32(F32(1.0) / s)
        x = (rng.uniform(-1, 1, 200_000) * amax).astype(F32)
        x[:1000] = (np.round(rng.uniform(-127, 127, 1000)) + 0.5).astype(F32) * s  # near ties
        assert np.array_equal(_adder_q(x, inv), _reference_q(x, inv))


def test_nan_maps_to_minus_127():
    x = np.array([np.nan], F32)
    assert _adder_q(x, F32(1.0))[0] == -127
