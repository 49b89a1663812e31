"""The GELU of the kernels (gelu_erf, esm-cpp_b200/csrc/epilogue.cuh) takes
erf(z) = sign(z) (1 - 2^(a R(a))), a = min(|z|, 4), R a degree-9 polynomial
fit of log2(erfc(a)) / a.  This CPU check evaluates the same float32 steps
(FMA Horner, ex2, the |z| > 4 cut) with the coefficients read from the
header and bounds the GELU against double-precision x/2 (1 + erf(x/sqrt 2))
by the op-level tolerance 1e-6 (1 + |gelu|) with a margin of ten."""
import math
import re
from pathlib import Path

import numpy as np

HDR = Path(__file__).resolve().parents[1] / "esm-cpp_b200" / "csrc" / "epilogue.cuh"


def _coeffs():
    text = HDR.read_text()
    body = re.search(r"constexpr float kR\[10\] = \{([^}]*)\}", text).group(1)
    return np.array([float.fromhex(v.strip().rstrip("f")) for v in body.split(",")], np.float32)


def _f32(v):
    return np.asarray(v, np.float64).astype(np.float32)


def _fma(a, b, c):
    return _f32(a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64))


def _gelu(x, kr):
    x = _f32(x)
    z = _f32(x * np.float32(0.70710678118654752440))
    az = np.abs(z)
    a = np.fmin(az, np.float32(4.0))
    r = np.full_like(a, kr[9])
    for c in kr[8::-1]:
        r = _fma(r, a, np.full_like(a, c))
    pen = np.fmax(_f32(az - np.float32(4.0)), np.float32(0.0))
    q = _fma(pen, np.full_like(a, -1.0e4), _f32(r * a))
    with np.errstate(over="ignore", under="ignore"):
        e = _f32(np.exp2(q.astype(np.float64)))
    e[e < 2.0 ** -126] = 0.0  # ftz
    erf_z = np.copysign(_f32(np.float32(1.0) - e), z)
    return _f32(_f32(x * np.float32(0.5)) * _f32(np.float32(1.0) + erf_z))


def test_gelu_within_a_tenth_of_op_tolerance():
    kr = _coeffs()
    rng = np.random.default_rng(3)
    x = np.concatenate([np.linspace(-12, 12, 400001), rng.standard_normal(300000) * 3,
                        [0.0, 1e-30, -1e-30, 5.656, -5.657, 40.0, -40.0, 1e4, -1e4]]).astype(np.float32)
    got = _gelu(x, kr).astype(np.float64)
    xd = x.astype(np.float64)
    ref = 0.5 * xd * (1.0 + np.array([math.erf(t / math.sqrt(2.0)) for t in xd]))
    assert (np.abs(got - ref) / (1.0 + np.abs(ref))).max() <= 1e-7


def test_gelu_special_values():
    kr = _coeffs()
    with np.errstate(invalid="ignore"):
        got = _gelu(np.array([0.0, np.inf, -np.inf, np.nan], np.float32), kr)
    assert got[0] == 0.0 and got[1] == np.inf and np.isnan(got[2]) and np.isnan(got[3])
