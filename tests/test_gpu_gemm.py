"""W8A8 INT8 GEMM on the tcgen05 tensor cores vs the oracle, through the C ABI.

Gates: int8 quantised activations and int32
accumulators bit-exact; dequantised outputs within rtol 1e-3 / atol 1 (they
are in fact bit-exact: the epilogue performs the reference's
FinalizeStore16 arithmetic, gemm_int8.cpp:109-126).  Shapes follow the
reference's Int8Shapes sweep (tests/cpp/test_gemm_shapes.cpp:147-217): row
tails, small M, N not a multiple of the tile, and the 650M shapes.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, N, K)
    (1, 16, 16), (7, 64, 48), (37, 96, 320), (128, 256, 128), (129, 200, 1280),
    (300, 3840, 1280), (513, 1280, 1280), (260, 5120, 1280), (257, 1280, 5120),
]


def _torch():
    import torch

    return torch


def _weights(rng, N, K, O):
    return O.quantize_weights((rng.standard_normal((N, K)) * 0.02).astype(np.float32))


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_quantize_and_int32_bitexact(cuda, O, M, N, K):
    from esm_b200 import ops

    torch = _torch()
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Wq, _ = _weights(rng, N, K, O)
    q, s = ops.quantize_activations(torch.from_numpy(A).to(cuda))
    acc = ops.gemm_int8_s32(q, torch.from_numpy(Wq).to(cuda))
    ops.synchronize()
    q_ref, s_ref = O.quantize_act_per_tensor(A)
    assert s.cpu().numpy()[0] == s_ref[0]
    assert np.array_equal(q.cpu().numpy()[:, :K], q_ref)
    assert np.array_equal(acc.cpu().numpy(), O.gemm_i8_s32(q_ref, Wq))


@pytest.mark.parametrize("M,N,K", SHAPES[:6])
def test_per_token_quantize_bitexact(cuda, O, M, N, K):
    from esm_b200 import ACT_PER_TOKEN, ops

    torch = _torch()
    rng = np.random.default_rng(M + 3 * N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    A[:, rng.integers(0, K, max(1, K // 100))] *= 20.0  # outlier channels
    q, s = ops.quantize_activations(torch.from_numpy(A).to(cuda), ACT_PER_TOKEN)
    ops.synchronize()
    q_ref, s_ref = O.quantize_act_per_token(A)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy()[:, :K], q_ref)


def _rounding_rows():
    """Rows whose absmax is 127, so the scale is exactly 1 and q = rne(x):
    every half-integer tie in [-127.5, 127.5], the bounds, values just off
    a tie, signed zeros and tiny values."""
    ties = np.arange(-127, 127, dtype=np.float32) + np.float32(0.5)
    extra = np.array([127.0, -127.0, 126.6, -126.4, 0.4999999, -0.5000001, 0.0, -0.0, 1e-30, -1e-30,
                      2.5, -2.5, 3.5, -3.5], np.float32)
    row = np.concatenate([ties, extra])
    return np.stack([row, row[::-1].copy(), -row, np.roll(row, 7)]).astype(np.float32)


@pytest.mark.parametrize("per_token", [False, True])
def test_activation_rounding_ties_bounds_and_nan(cuda, O, per_token):
    """The quantisers round in the float adder (x * inv + 1.5 * 2^23): ties go
    to even exactly as the reference's conversion, the bounds are kept, and a
    NaN maps to -127 (the reference's AVX-512 conversion gives INT_MIN, then
    the clamp)."""
    from esm_b200 import ACT_PER_TENSOR, ACT_PER_TOKEN, ops

    torch = _torch()
    A = _rounding_rows()
    mode = ACT_PER_TOKEN if per_token else ACT_PER_TENSOR
    q, s = ops.quantize_activations(torch.from_numpy(A).to(cuda), mode)
    ops.synchronize()
    q_ref, s_ref = O.quantize_act_per_token(A) if per_token else O.quantize_act_per_tensor(A)
    assert np.all(s.cpu().numpy() == 1.0) and np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy()[:, :A.shape[1]], q_ref)
    assert np.array_equal(q_ref[0, :254], np.rint(A[0, :254]).astype(np.int8))
    An = A.copy()
    An[:, 5] = np.nan
    qn, sn = ops.quantize_activations(torch.from_numpy(An).to(cuda), mode)
    ops.synchronize()
    qn = qn.cpu().numpy()[:, :A.shape[1]]
    assert np.all(qn[:, 5] == -127)
    keep = np.arange(A.shape[1]) != 5
    assert np.array_equal(qn[:, keep], q_ref[:, keep])
    assert np.all(sn.cpu().numpy() == 1.0)


@pytest.mark.parametrize("per_token", [False, True])
@pytest.mark.parametrize("M,N,K", SHAPES + [(33, 48, 40), (5, 17, 23)])
def test_linear_int8_matches_oracle(cuda, O, M, N, K, per_token):
    from esm_b200 import ACT_PER_TENSOR, ACT_PER_TOKEN, ops

    torch = _torch()
    rng = np.random.default_rng(M * 13 + N * 5 + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Wq, ws = _weights(rng, N, K, O)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    C = ops.linear_int8(torch.from_numpy(A).to(cuda), torch.from_numpy(Wq).to(cuda),
                        torch.from_numpy(ws).to(cuda), torch.from_numpy(bias).to(cuda),
                        ACT_PER_TOKEN if per_token else ACT_PER_TENSOR)
    ops.synchronize()
    want = O.linear_int8(A, Wq, ws, bias, per_token=per_token)
    got = C.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1.0)
    assert np.array_equal(got, want), "epilogue should reproduce FinalizeStore16 exactly"


def test_linear_int8_matches_reference_vnni(cuda, O, R):
    """Against the reference's own LinearVnni (one activation scale over M)."""
    from esm_b200 import ops

    torch = _torch()
    rng = np.random.default_rng(11)
    M, N, K = 96, 1280, 1280
    A = rng.standard_normal((M, K)).astype(np.float32)
    Wq, ws = _weights(rng, N, K, O)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    want = np.zeros((M, N), np.float32)
    O.ref_check(R.ref_linear_int8_vnni(A.ctypes.data, Wq.ctypes.data, ws.ctypes.data,
                                       bias.ctypes.data, want.ctypes.data, M, N, K))
    C = ops.linear_int8(torch.from_numpy(A).to(cuda), torch.from_numpy(Wq).to(cuda),
                        torch.from_numpy(ws).to(cuda), torch.from_numpy(bias).to(cuda))
    ops.synchronize()
    assert np.array_equal(C.cpu().numpy(), want)


@pytest.mark.parametrize("N,K", [(3840, 1280), (1280, 1280), (5120, 1280), (1280, 5120)])
def test_config2_full_size_sampled_rows(cuda, O, N, K):
    """Config 2 at M = 32768 with 1% x20 outlier channels; int32 accumulators
    of 64 sampled rows bit-exact, and every row's int8 quantisation exact."""
    from esm_b200 import ops

    torch = _torch()
    M = 32768
    g = torch.Generator(device=cuda).manual_seed(N + K)
    A = torch.randn((M, K), device=cuda, generator=g)
    cols = torch.randperm(K, device=cuda, generator=g)[: K // 100]
    A[:, cols] *= 20.0
    rng = np.random.default_rng(N * K)
    Wq, _ = _weights(rng, N, K, O)
    q, s = ops.quantize_activations(A)
    acc = ops.gemm_int8_s32(q, torch.from_numpy(Wq).to(cuda))
    ops.synchronize()
    A_h = A.cpu().numpy()
    q_ref, s_ref = O.quantize_act_per_tensor(A_h)
    assert s.cpu().numpy()[0] == s_ref[0]
    assert np.array_equal(q.cpu().numpy(), q_ref)
    rows = np.sort(rng.choice(M, 64, replace=False))
    assert np.array_equal(acc.cpu().numpy()[rows], O.gemm_i8_s32(q_ref[rows], Wq))


@pytest.mark.parametrize("N,K", [(1, 1), (7, 33), (257, 1000), (3840, 1280)])
def test_quantize_weights_on_device_bit_exact(cuda, O, N, K):
    """esmcu_quantize_weights = quant::Quantize (pack.cpp:149-177): codes and
    scales bit-identical to the numpy restatement and the oracle's C one,
    including all-zero rows (scale 0), rounding ties and outlier rows."""
    import torch

    from esm_b200 import ops
    from esm_b200.prep import quantize_weight

    rng = np.random.default_rng(N * 31 + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[:: max(N // 3, 1)] *= 50.0                      # outlier rows
    if N > 2:
        W[1] = 0.0                                    # all-zero row
        W[2, :] = np.float32(1.0)                     # ties: w * inv = 127 exactly
        W[2, :: 2] = np.float32(0.5 / 127.0)           # and a half-step (rne)
    q, s = ops.quantize_weights(torch.from_numpy(W).to(cuda))
    q, s = q.cpu().numpy(), s.cpu().numpy()
    qh, sh = quantize_weight(W)
    qo, so = O.quantize_weights(W)
    assert np.array_equal(q, qh) and np.array_equal(s, sh)
    assert np.array_equal(q, qo) and np.array_equal(s, so)


def test_model_quantize_weights_on_device_matches_host(cuda):
    from esm_b200 import synth

    arch = dict(num_hidden_layers=2, hidden_size=128, num_attention_heads=2, head_dim=64,
                intermediate_size=512)
    a, b = synth.random_model(arch, seed=61), synth.random_model(arch, seed=61)
    a.quantize_weights()
    b.quantize_weights(on_device=True)
    for la, lb in zip(a.layers, b.layers):
        for n in ("q", "k", "v", "out", "fc1", "fc2"):
            assert np.array_equal(la[n + "_wq"], lb[n + "_wq"])
            assert np.array_equal(la[n + "_ws"], lb[n + "_ws"])
    a.close()
    b.close()
