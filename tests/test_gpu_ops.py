"""Kernel-facade ops on the GPU vs the oracle (and the compiled reference),
through the C ABI: LayerNorm, GELU, residual, scale, RoPE, varlen attention,
FP32 Linear.  Tolerances are the reference's own precision classes
(tests/cpp/test_gemm_shapes.cpp:250-256, test_attention_varlen.cpp:374-375):
FP32 1e-4 * (1 + |ref|)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _close(got, want, tol=1e-4):
    err = np.abs(got - want) / (1.0 + np.abs(want))
    assert err.max() <= tol, f"max rel err {err.max():.3e}"


@pytest.mark.parametrize("rows,d", [(1, 320), (37, 1280), (1000, 1280), (64, 2560), (5, 100)])
def test_layernorm_matches_ref_twin(cuda, O, rows, d):
    from esm_b200 import ops

    rng = np.random.default_rng(rows + d)
    x = (rng.standard_normal((rows, d)) * 3 + 0.5).astype(np.float32)
    g = rng.standard_normal(d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    y = ops.layernorm(_t(x, cuda), _t(g, cuda), _t(b, cuda))
    ops.synchronize()
    got, want = y.cpu().numpy(), O.layernorm(x, g, b)
    # Double-precision sums make the float result the reference's (LayerNormRef)
    # except when a sum rounds across a float boundary: allow rare 1-ulp cases.
    mism = np.mean(got != want)
    assert mism < 1e-3, f"{mism:.2e} of outputs differ from LayerNormRef"
    _close(got, want, 1e-6)


def test_layernorm_known_answer(cuda):
    """tests/cpp/test_kernels.cpp:113-139: x = [1,2,3,4], gamma 1, beta 0."""
    from esm_b200 import ops

    x = np.array([[1, 2, 3, 4]], np.float32)
    y = ops.layernorm(_t(x, cuda), _t(np.ones(4, np.float32), cuda), _t(np.zeros(4, np.float32), cuda))
    ops.synchronize()
    mean, var = 2.5, 1.25
    want = (x - mean) / np.sqrt(var + 1e-5)
    np.testing.assert_allclose(y.cpu().numpy(), want, atol=1e-5)


def test_gelu_known_answers_and_oracle(cuda, O):
    from esm_b200 import ops

    x = np.array([1.0, -1.0, 2.0], np.float32)
    y = ops.gelu(_t(x, cuda))
    ops.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), [0.8413447, -0.1586553, 1.9544997], atol=1e-6)
    xs = (np.random.default_rng(1).standard_normal(100000) * 4).astype(np.float32)
    y = ops.gelu(_t(xs, cuda))
    ops.synchronize()
    _close(y.cpu().numpy(), O.gelu(xs), 1e-6)


def test_residual_and_scale_exact(cuda):
    from esm_b200 import ops

    rng = np.random.default_rng(2)
    a = rng.standard_normal(10001).astype(np.float32)
    b = rng.standard_normal(10001).astype(np.float32)
    ta = _t(a, cuda)
    ops.residual_add_inplace(ta, _t(b, cuda))
    ops.scale_inplace(ta, 0.125)
    ops.synchronize()
    assert np.array_equal(ta.cpu().numpy(), ((a + b) * np.float32(0.125)).astype(np.float32))


def test_rope_tables_bitexact(O):
    from esm_b200 import ops

    for L, dh in [(300, 64), (1024, 16), (5, 32)]:
        c, s = ops.rope_build_tables(L, dh)
        co, so = O.rope_build_tables(L, dh)
        assert np.array_equal(c, co) and np.array_equal(s, so)


def test_rope_varlen_positions_restart(cuda, O):
    """rope.cpp AVX-512 form, bit-exact; positions restart per sequence
    (tests/cpp/test_attention_varlen.cpp:144-183)."""
    from esm_b200 import ops

    rng = np.random.default_rng(3)
    cu = np.array([0, 5, 5, 30, 31, 100], np.int32)
    H, dh = 3, 64
    x = rng.standard_normal((100, H, dh)).astype(np.float32)
    c, s = ops.rope_build_tables(128, dh)
    tx = _t(x, cuda)
    ops.rope_apply_varlen(tx, _t(c, cuda), _t(s, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    want = O.rope_apply_varlen(x, c, s, cu, H, dh, fused=True)
    assert np.array_equal(tx.cpu().numpy(), want)
    # position 0 of every sequence is the identity rotation
    for b in range(len(cu) - 1):
        if cu[b + 1] > cu[b]:
            assert np.array_equal(tx.cpu().numpy()[cu[b]], x[cu[b]])


# head_dim 64 runs three tensor-core kernels by length: <= 128, 129..256 and
# > 256 (128-row query tiles, keys in 128-key blocks; the last block ragged).
@pytest.mark.parametrize("lens,H,dh", [([1], 1, 16), ([7, 13, 1], 2, 16), ([33, 250, 90], 20, 64),
                                       ([129, 300], 4, 64), ([1024], 2, 64), ([17, 5], 3, 32),
                                       ([402, 3, 257, 130, 513], 20, 64), ([700, 1000, 260], 3, 64),
                                       ([1500, 384, 385], 2, 64)])
def test_attention_varlen_matches_oracle(cuda, O, lens, H, dh):
    from esm_b200 import ops

    rng = np.random.default_rng(sum(lens) + H)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q, k, v = (rng.standard_normal((3, T, H, dh)).astype(np.float32))
    q *= np.float32(1.0 / np.sqrt(dh))
    out = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    _close(out.cpu().numpy(), O.attention_varlen(q, k, v, cu, H, dh))


def test_attention_bf16_mode_matches_oracle(cuda, O, monkeypatch):
    """ESM_AMX_ATTENTION=on (attention.cpp:686-700): Q and K rounded to bf16
    (round to nearest even) before the scores, on all three tensor-core
    kernels (<= 128, 129..256, > 256 tokens); S then needs one tf32 MMA
    per k-step.  head_dim 16 is not a multiple of 32 and stays FP32, as in
    the reference.  The caller's q and k are not modified."""
    from esm_b200 import ops

    monkeypatch.setenv("ESM_AMX_ATTENTION", "on")
    rng = np.random.default_rng(71)
    for lens, H, dh in (([90, 3, 200, 402, 129, 1], 8, 64), ([33, 70], 2, 16)):
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        T = int(cu[-1])
        q, k, v = (rng.standard_normal((3, T, H, dh)).astype(np.float32))
        q *= np.float32(1.0 / np.sqrt(dh))
        tq, tk = _t(q, cuda), _t(k, cuda)
        out = ops.attention_varlen(tq, tk, _t(v, cuda), _t(cu, cuda), H, dh)
        ops.synchronize()
        assert np.array_equal(tq.cpu().numpy(), q) and np.array_equal(tk.cpu().numpy(), k)
        bf16 = dh % 32 == 0
        _close(out.cpu().numpy(), O.attention_varlen(q, k, v, cu, H, dh, bf16=bf16))
        if bf16:
            assert np.abs(out.cpu().numpy() - O.attention_varlen(q, k, v, cu, H, dh)).max() > 1e-4


def test_attention_matches_reference_avx512(cuda, O, R):
    from esm_b200 import ops

    rng = np.random.default_rng(9)
    lens = [122, 90, 250, 17]
    H, dh = 20, 64
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q, k, v = (rng.standard_normal((3, T, H, dh)).astype(np.float32))
    want = np.zeros_like(q)
    O.ref_check(R.ref_attention_varlen(q.ctypes.data, k.ctypes.data, v.ctypes.data, cu.ctypes.data,
                                       len(lens), H, dh, want.ctypes.data))
    out = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    _close(out.cpu().numpy(), want)


def test_attention_isolation_poisoned_kv(cuda):
    """tests/cpp/test_attention_varlen.cpp:185-225: poisoning sequence 2's
    K/V must not change sequence 1's output."""
    from esm_b200 import ops

    rng = np.random.default_rng(5)
    cu = np.array([0, 40, 100], np.int32)
    H, dh = 4, 64
    q, k, v = (rng.standard_normal((3, 100, H, dh)).astype(np.float32))
    a = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    k2, v2 = k.copy(), v.copy()
    k2[40:] = 1e4
    v2[40:] = -1e4
    b = ops.attention_varlen(_t(q, cuda), _t(k2, cuda), _t(v2, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    assert np.array_equal(a.cpu().numpy()[:40], b.cpu().numpy()[:40])


def test_attention_isolation_long_sequences(cuda):
    """The same property across the > 256 kernel's ragged last key block and
    query tile: sequence 1 (300 tokens) shares its last 128-row tiles with
    sequence 2, whose K/V are poisoned."""
    from esm_b200 import ops

    rng = np.random.default_rng(6)
    cu = np.array([0, 300, 700], np.int32)
    H, dh = 2, 64
    q, k, v = (rng.standard_normal((3, 700, H, dh)).astype(np.float32))
    a = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    k2, v2 = k.copy(), v.copy()
    k2[300:] = 1e4
    v2[300:] = -1e4
    b = ops.attention_varlen(_t(q, cuda), _t(k2, cuda), _t(v2, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    assert np.array_equal(a.cpu().numpy()[:300], b.cpu().numpy()[:300])


@pytest.mark.parametrize("late", [1, 3])
def test_attention_long_late_block_max(cuda, O, late):
    """The > 256 kernel's reference point starts at the first key block's row
    max; here key block `late` scores far above block 0 for every query row
    (keys aligned with the common direction of q), which moves it and
    rescales O and the row sums mid-sequence.  The result must still match
    the oracle's max-first softmax."""
    from esm_b200 import ops

    rng = np.random.default_rng(40 + late)
    L, H, dh = 600, 2, 64
    cu = np.array([0, L], np.int32)
    q = (0.125 * (1.0 + 0.1 * rng.standard_normal((L, H, dh)))).astype(np.float32)
    k = rng.standard_normal((L, H, dh)).astype(np.float32)
    v = rng.standard_normal((L, H, dh)).astype(np.float32)
    # block `late` (keys 128 late ..): scores about 8 * 2 = 16 against about 0 +- 3 elsewhere
    k[128 * late:128 * late + 40] = np.float32(2.0) + 0.05 * rng.standard_normal((40, H, dh)).astype(np.float32)
    out = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), H, dh)
    ops.synchronize()
    _close(out.cpu().numpy(), O.attention_varlen(q, k, v, cu, H, dh))


@pytest.mark.parametrize("L", [64, 600])
def test_attention_large_scores_finite(cuda, L):
    """Scores of 57600 (q = k = 30): the softmax's row max keeps every
    exponential finite; uniform weights give the mean of V."""
    from esm_b200 import ops

    cu = np.array([0, L], np.int32)
    q = np.full((L, 1, 64), 30.0, np.float32)
    k = np.full((L, 1, 64), 30.0, np.float32)
    v = np.random.default_rng(0).standard_normal((L, 1, 64)).astype(np.float32)
    out = ops.attention_varlen(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), 1, 64)
    ops.synchronize()
    o = out.cpu().numpy()
    assert np.isfinite(o).all()
    np.testing.assert_allclose(o[0, 0], v.mean(axis=0)[0], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(o[L - 1, 0], v.mean(axis=0)[0], rtol=1e-4, atol=1e-5)


# K % 4 == 0 takes the 3xTF32 tensor-core path (BN = 128 tiles, or CTA pairs
# when there are >= 74 pair tiles: the 1200 x 4096 case), else FP32 SIMT
# (K = 37).
@pytest.mark.parametrize("M,N,K", [(1, 33, 320), (130, 1280, 1280), (77, 33, 1280), (9, 11, 40),
                                   (1200, 4096, 500), (300, 1000, 1284), (50, 70, 37)])
def test_linear_f32_matches_oracle(cuda, O, M, N, K):
    from esm_b200 import ops

    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    C = ops.linear(_t(A, cuda), _t(W, cuda), _t(b, cuda))
    ops.synchronize()
    _close(C.cpu().numpy(), O.linear_f32(A, W, b))
