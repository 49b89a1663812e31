"""The reference-rounding mode (esmcu_math_mode ESMCU_MATH_AVX512) op by op:
LayerNorm, GELU and varlen attention on the GPU against the oracle's
restatement of the reference's default x86 kernels (itself pinned bit for bit
to the compiled reference in test_oracle_avx.py).  The gate is bit equality.
Whole-forward checks of the mode are in test_gpu_650m.py and test_gpu_3b.py.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture
def avx(cuda):
    from esm_b200 import ops

    ops.set_math_mode("avx512")
    yield
    ops.set_math_mode("default")


@pytest.mark.parametrize("rows,d", [(1, 320), (333, 1280), (64, 2560), (40, 480), (9, 16)])
def test_layernorm_avx_bit_exact(avx, cuda, O, rows, d):
    from esm_b200 import ops

    rng = np.random.default_rng(rows + d)
    x = (rng.standard_normal((rows, d)) * 3 + 0.5).astype(np.float32)
    g = rng.standard_normal(d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    y = ops.layernorm(_t(x, cuda), _t(g, cuda), _t(b, cuda))
    ops.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(O.layernorm_avx(x, g, b)))


def test_gelu_avx_bit_exact(avx, cuda, O):
    from esm_b200 import ops

    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(1_000_000) * 4, np.linspace(-13, 13, 4001),
                        [0.0, -0.0, 1e-30]]).astype(np.float32)
    y = ops.gelu(_t(x, cuda))
    ops.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(O.gelu_avx(x)))


@pytest.mark.parametrize("lens,H,dh", [([122, 90, 250, 17, 1, 16, 33, 31], 20, 64), ([402, 129], 4, 64),
                                       ([50, 7, 64], 3, 16), ([100, 5], 2, 32), ([1000], 1, 64)])
def test_attention_avx_bit_exact(avx, cuda, O, lens, H, dh):
    from esm_b200 import ops

    rng = np.random.default_rng(sum(lens) + H)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q, k, v = rng.standard_normal((3, T, H, dh)).astype(np.float32)
    q *= np.float32(1.0 / np.sqrt(dh))
    out = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(O.attention_avx(q, k, v, cu, H, dh)))


def test_mode_rejects_unsupported_shapes(avx, cuda):
    from esm_b200 import EsmCudaError, _lib, ops

    x = _t(np.ones((4, 24), np.float32), cuda)
    g = _t(np.ones(24, np.float32), cuda)
    with pytest.raises(EsmCudaError) as ei:
        ops.layernorm(x, g, g)
    assert _lib.STATUS[ei.value.code] == "INVALID_ARGUMENT"
