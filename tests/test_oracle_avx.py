"""The oracle's restatement of the reference's default x86 kernels (the
AVX-512 LayerNorm, GELU and varlen attention that its dispatch runs on this
hardware, plus the C library's expf that the attention calls past whole
16-key blocks) against the reference compiled from its own sources and the
host C library, bit for bit, on the CPU.  These pin the checker of the GPU's
reference-rounding mode (esmcu_math_mode ESMCU_MATH_AVX512)."""
import ctypes as C

import numpy as np
import pytest


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("d", [320, 480, 640, 1280, 2560, 16, 48])
def test_layernorm_avx_matches_reference(O, R, d):
    rng = np.random.default_rng(d)
    x = (rng.standard_normal((97, d)) * 3 + 0.7).astype(np.float32)
    x[5] = 0.0
    x[7] *= np.float32(1e4)
    g = rng.standard_normal(d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    want = np.zeros_like(x)
    O.ref_check(R.ref_layernorm(x.ctypes.data, g.ctypes.data, b.ctypes.data, C.c_float(1e-5),
                                want.ctypes.data, x.shape[0], d))
    assert np.array_equal(_bits(O.layernorm_avx(x, g, b)), _bits(want))


def test_gelu_avx_matches_reference(O, R):
    rng = np.random.default_rng(2)
    x = np.concatenate([(rng.standard_normal(500_000) * 4), np.linspace(-13, 13, 20001),
                        [0.0, -0.0, 1e-30, -1e-30, 13.0, -13.0]]).astype(np.float32)
    want = np.zeros_like(x)
    O.ref_check(R.ref_gelu(x.ctypes.data, want.ctypes.data, x.size))
    assert np.array_equal(_bits(O.gelu_avx(x)), _bits(want))


def test_expf_libc_matches_host_c_library(O):
    libm = C.CDLL("libm.so.6")
    libm.expf.restype, libm.expf.argtypes = C.c_float, [C.c_float]
    rng = np.random.default_rng(3)
    x = np.concatenate([-rng.exponential(4.0, 60_000), -rng.random(20_000) * 110,
                        rng.standard_normal(5_000) * 30,
                        [0.0, -0.0, -87.33, -103.2, -103.97, -104.0, 88.5, -np.inf]]).astype(np.float32)
    want = np.array([libm.expf(float(v)) for v in x], np.float32)
    assert np.array_equal(_bits(O.expf_libc(x)), _bits(want))


@pytest.mark.parametrize("lens,H,dh", [([122, 90, 250, 17, 1, 16, 33], 4, 64), ([50, 7, 32], 2, 16),
                                       ([100, 64, 3], 3, 32), ([402, 129], 2, 64)])
def test_attention_avx_matches_reference(O, R, lens, H, dh):
    rng = np.random.default_rng(sum(lens) + dh)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q, k, v = rng.standard_normal((3, T, H, dh)).astype(np.float32)
    q *= np.float32(1.0 / np.sqrt(dh))
    want = np.zeros_like(q)
    O.ref_check(R.ref_attention_varlen(q.ctypes.data, k.ctypes.data, v.ctypes.data, cu.ctypes.data,
                                       len(lens), H, dh, want.ctypes.data))
    assert np.array_equal(_bits(O.attention_avx(q, k, v, cu, H, dh)), _bits(want))
