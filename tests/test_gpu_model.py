"""End-to-end packed-varlen forward on the GPU vs the oracle and the reference.

Mirrors the reference's Python integration tests (tests/python/
test_forward_packed.py:42-149, test_forward_scheduled.py:35-96) with
random-init weights (no HF checkpoints exist here).  Gates:
  FP32 models: logits within 1e-4 * (1 + |ref|) (and Pearson >= 0.99999).
  W8A8 models: every int8 code and int32 accumulator is bit-exact at the op
  level (test_gpu_gemm.py); over a whole forward, last-ulp differences of
  the FP32 ops (LN sums, attention, GELU) flip single int8 roundings and the
  flips compound, exactly as between the reference's own VNNI and AMX paths.
  The whole-forward W8A8 gate is therefore per-sequence Pearson >= 0.9999
  plus an absolute bound (the reference agrees with itself across ISAs to
  Pearson ~0.999 at 650M, see test_gpu_650m.py).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TINY = dict(num_hidden_layers=2, hidden_size=128, num_attention_heads=2, head_dim=64,
            intermediate_size=512)


def _close(got, want, tol=1e-4):
    err = np.abs(got - want) / (1.0 + np.abs(want))
    assert err.max() <= tol, f"max rel err {err.max():.3e}"


W8A8_PEARSON = 0.9999
# One flipped int8 code moves a tiny model's logits by ~1e-2.
W8A8_ATOL = 5e-2


def _pearson_each(got, want, cu, thr=W8A8_PEARSON):
    for b in range(len(cu) - 1):
        g, w = got[cu[b]:cu[b + 1]].ravel(), want[cu[b]:cu[b + 1]].ravel()
        if g.size > 1:
            r = np.corrcoef(g, w)[0, 1]
            assert r >= thr, f"sequence {b}: Pearson {r:.7f}"


@pytest.fixture(scope="module")
def tiny_fp32(cuda):
    from esm_b200 import synth

    m = synth.random_model(TINY, seed=1)
    yield m
    m.close()


@pytest.fixture(scope="module")
def tiny_q8(cuda):
    from esm_b200 import synth

    m = synth.random_model(TINY, seed=2)
    stats = m.calibrate(synth.residue_ids([40, 60, 90], seed=3))
    m.apply_smoothquant(stats, 0.5)
    m.quantize_weights()
    yield m
    m.close()


def _batch(lens, seed):
    from esm_b200 import synth

    seqs = synth.residue_ids(lens, seed=seed)
    ids, cu = synth.pack(seqs)
    return seqs, ids, cu


def test_fp32_packed_matches_oracle(tiny_fp32, O):
    seqs, ids, cu = _batch([3, 40, 1, 120, 250], 5)
    got = tiny_fp32.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(tiny_fp32, ids, cu)
    _close(got, want)
    _pearson_each(got, want, cu, 0.99999)


def test_fp32_packed_matches_reference(tiny_fp32, O, R, tmp_path):
    p = tmp_path / "tiny.safetensors"
    tiny_fp32.save_to_safetensors(p)
    ref = O.RefModel(p)
    seqs, ids, cu = _batch([30, 7, 66], 6)
    got = tiny_fp32.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    _close(got, ref.forward_packed(ids, cu))


def test_w8a8_packed_matches_oracle(tiny_q8, O):
    seqs, ids, cu = _batch([12, 50, 3, 90], 7)
    got = tiny_q8.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(tiny_q8, ids, cu)
    _pearson_each(got, want, cu)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)


def test_w8a8_packed_matches_reference_via_gguf(tiny_q8, O, R, tmp_path):
    p = tmp_path / "tiny_q8.gguf"
    tiny_q8.save_to_gguf(p)
    ref = O.RefModel(p)
    assert ref.quantized == 1
    O.ref_force_isa("avx512vnni")  # one activation scale over all rows
    try:
        seqs, ids, cu = _batch([12, 50, 3, 90, 200], 8)
        want = ref.forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    got = tiny_q8.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    _pearson_each(got, want, cu)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)


def test_fp32_hidden_states_match_reference(tiny_fp32, O, R, tmp_path):
    """forward_with_hidden_states (the reference's binding, _core.cpp:511-524;
    test_against_hf.py:100-125 checks the same N+1 states against HF): every
    hidden state and the logits within the FP32 class of the reference's own
    ForwardWithHiddenStates."""
    p = tmp_path / "tiny_h.safetensors"
    tiny_fp32.save_to_safetensors(p)
    ref = O.RefModel(p)
    ids = _batch([57], 11)[0][0]
    logits, hidden = tiny_fp32.forward_with_hidden_states(ids)
    want_logits, want_hidden = ref.forward_hidden(ids)
    assert len(hidden) == TINY["num_hidden_layers"] + 1
    for j in range(len(hidden)):
        assert hidden[j].shape == (ids.size, TINY["hidden_size"])
        _close(hidden[j], want_hidden[j])
    _close(logits, want_logits)


def test_hidden_states_packed_match_oracle_and_single(tiny_fp32, tiny_q8, O):
    """The packed form (hidden_packed_out of ForwardPackedInto): the FP32
    model matches the oracle's packed forward to the FP32 class and each
    sequence's rows match its single-sequence call (1e-5); the W8A8
    model matches the oracle under the whole-forward W8A8 gate."""
    seqs, ids, cu = _batch([20, 64, 5], 12)
    L1 = TINY["num_hidden_layers"] + 1
    logits, hidden = tiny_fp32.forward_packed_hidden_states(ids, cu)
    want = []
    want_logits = O.forward_packed(tiny_fp32, ids, cu, hidden=want)
    assert hidden.shape == (L1, ids.size, TINY["hidden_size"]) and len(want) == L1
    for j in range(L1):
        _close(hidden[j], want[j])
    _close(logits, want_logits)
    for b, s in enumerate(seqs):
        _, hs = tiny_fp32.forward_with_hidden_states(s)
        for j in range(L1):
            _close(hidden[j][cu[b]:cu[b + 1]], hs[j], tol=1e-5)
    lq, hq = tiny_q8.forward_packed_hidden_states(ids, cu)
    wq = []
    O.forward_packed(tiny_q8, ids, cu, hidden=wq)
    assert np.array_equal(hq[0], wq[0])  # the embedding is exact
    for j in range(1, L1):
        np.testing.assert_allclose(hq[j], wq[j], rtol=1e-3, atol=W8A8_ATOL)
        r = np.corrcoef(hq[j].ravel(), wq[j].ravel())[0, 1]
        assert r >= W8A8_PEARSON, f"hidden state {j}: Pearson {r:.7f}"


def test_gguf_round_trip_of_reference_artefact(tiny_fp32, O, R, tmp_path):
    """The reference calibrates, migrates, quantises and saves a Q8_ESM GGUF
    (quantize.py:35-91); this package loads it and matches the reference's
    forward on it."""
    from esm_b200 import Model, synth

    st = tmp_path / "m.safetensors"
    tiny_fp32.save_to_safetensors(st)
    ref = O.RefModel(st)
    ref.calibrate_smoothquant(synth.residue_ids([20, 40], seed=9), 99.9, 0.5)
    ref.quantize()
    gg = tmp_path / "m_q8.gguf"
    ref.save_gguf(gg)
    m = Model.load(gg)
    assert m.config.weights_quantized
    seqs, ids, cu = _batch([25, 80, 11], 10)
    O.ref_force_isa("avx512vnni")
    try:
        want = O.RefModel(gg).forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    _pearson_each(got, want, cu)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)
    m.close()


def test_packed_equals_serial_fp32(tiny_fp32):
    """test_forward_packed.py:42-69."""
    seqs, ids, cu = _batch([9, 31, 64], 11)
    packed = tiny_fp32.forward_packed(ids, cu)
    for s, p in zip(seqs, packed):
        _close(p, tiny_fp32.forward(s))


def test_mask_ratio_isolation(tiny_fp32):
    """test_forward_packed.py:85-117: masking tokens in sequence 0 leaves
    sequence 1's logits unchanged (per-sequence token-dropout rescale)."""
    from esm_b200 import MASK_ID

    seqs, ids, cu = _batch([20, 30], 12)
    a = tiny_fp32.forward_packed(ids, cu)
    ids2 = ids.copy()
    ids2[3:8] = MASK_ID
    b = tiny_fp32.forward_packed(ids2, cu)
    assert np.array_equal(a[1], b[1])
    assert not np.array_equal(a[0], b[0])


def test_pad_masks_zero_rows_match_reference(tiny_fp32, O, R, tmp_path):
    p = tmp_path / "tiny.safetensors"
    tiny_fp32.save_to_safetensors(p)
    ref = O.RefModel(p)
    seqs, ids, cu = _batch([10, 15], 13)
    masks = np.ones_like(ids)
    masks[9:12] = 0
    got = np.concatenate(tiny_fp32.forward_packed(ids, cu, masks))
    _close(got, ref.forward_packed(ids, cu, masks))


def test_validation_errors(tiny_fp32):
    from esm_b200 import EsmCudaError

    ids = np.array([0, 5, 6, 2], np.int32)
    with pytest.raises(EsmCudaError, match="cu_seqlens\\[0\\] must be 0"):
        tiny_fp32.forward_packed(ids, np.array([1, 4], np.int32))
    with pytest.raises(EsmCudaError, match="non-decreasing"):
        tiny_fp32.forward_packed(ids, np.array([0, 3, 2, 4], np.int32))
    with pytest.raises(EsmCudaError, match="must equal packed_ids.size"):
        tiny_fp32.forward_packed(ids, np.array([0, 3], np.int32))
    with pytest.raises(EsmCudaError, match="out of range"):
        tiny_fp32.forward_packed(np.array([0, 99], np.int32), np.array([0, 2], np.int32))
    assert tiny_fp32.forward(np.zeros(0, np.int32)).shape == (0, 33)


def test_forward_scheduled_matches_reference(tiny_q8, O, R, tmp_path):
    """test_forward_scheduled.py:35-96: caller order kept, groups from
    PlanBatches, each group's numerics equal to the reference's."""
    from esm_b200 import synth

    p = tmp_path / "q8.gguf"
    tiny_q8.save_to_gguf(p)
    ref = O.RefModel(p)
    lens = synth.varlen_lengths(40, seed=14, mean=60, sd=40, lo=5, hi=200)
    seqs = synth.residue_ids(lens, seed=15)
    O.ref_force_isa("avx512vnni")
    try:
        want = ref.forward_scheduled(seqs, 1.2, 16)
    finally:
        O.ref_force_isa(None)
    got = tiny_q8.forward_scheduled(seqs, imbalance_threshold=1.2, max_batch_size=16)
    assert [g.shape for g in got] == [(len(s), 33) for s in seqs]
    for g, w in zip(got, want):
        if g.size > 33:
            r = np.corrcoef(g.ravel(), w.ravel())[0, 1]
            assert r >= W8A8_PEARSON
        np.testing.assert_allclose(g, w, rtol=1e-3, atol=W8A8_ATOL)


def test_per_token_mode_matches_oracle(cuda, O):
    from esm_b200 import synth

    m = synth.random_model(TINY, seed=16)
    m.quantize_weights()
    m.set_act_quant("per_token")
    seqs, ids, cu = _batch([17, 40, 2], 17)
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(m, ids, cu, per_token=True)
    _pearson_each(got, want, cu)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)
    m.close()


def test_config0_esm2_8m_fp32_matches_reference(cuda, O, R, tmp_path):
    """8M FP32, 64 sequences, residues U[32,256], vs the
    reference's ForwardScheduled on the same safetensors."""
    from esm_b200 import synth

    m = synth.random_model("esm2_8m", seed=0)
    p = tmp_path / "8m.safetensors"
    m.save_to_safetensors(p)
    ref = O.RefModel(p)
    seqs = synth.residue_ids(synth.uniform_lengths(64, 0, 32, 256), seed=0)
    want = ref.forward_scheduled(seqs)
    got = m.forward_scheduled(seqs)
    for g, w in zip(got, want):
        _close(g, w)
    m.close()


def test_multi_replica_dispatch_matches_single(tiny_q8):
    """esmcu_forward_scheduled_multi with two replicas (both on device 0 here)
    returns the single-replica result in caller order."""
    from esm_b200 import Model, forward_scheduled_multi, synth

    other = Model(tiny_q8.config, tiny_q8.embed, tiny_q8.layers, tiny_q8.head, device=0)
    seqs = synth.residue_ids(synth.varlen_lengths(30, seed=18, mean=50, sd=30, lo=3, hi=150), seed=19)
    want = tiny_q8.forward_scheduled(seqs, max_batch_size=8)
    got = forward_scheduled_multi([tiny_q8, other], seqs, max_batch_size=8)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    other.close()


def test_int8_lm_head_matches_oracle_and_reference(O, R, tmp_path, monkeypatch, cuda):
    """ESM_QUANTIZE_LM_HEAD=on (model.cpp:1487-1492): lm_head.dense runs as
    LinearInt8 (model.cpp:1209-1211) through esmcu_model_set_head_int8.  The
    device forward matches the oracle and the compiled reference under the
    whole-forward W8A8 gate; the masked-marginal head (scored rows only,
    activation scale still over all T rows) matches the full logits' rows."""
    from esm_b200 import Model, synth

    st = tmp_path / "tiny_lm8.safetensors"
    synth.random_model(TINY, seed=31).save_to_safetensors(st)
    seqs, ids, cu = _batch([40, 3, 130, 250], 32)
    monkeypatch.setenv("ESM_QUANTIZE_LM_HEAD", "on")
    m = Model.load(st)
    m.quantize_weights()
    assert m.config.lm_head_dense_quantized
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(m, ids, cu)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)
    _pearson_each(got, want, cu)
    ref = O.RefModel(st)
    ref.quantize()
    O.ref_force_isa("avx512vnni")
    try:
        rw = ref.forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    np.testing.assert_allclose(got, rw, rtol=1e-3, atol=W8A8_ATOL)
    _pearson_each(got, rw, cu)
    rows = np.array([5, 1, 64, 249], np.int32)
    lp = m.masked_marginals(seqs, rows)
    full = m.forward_scheduled(seqs)
    x = np.stack([full[i][r] for i, r in enumerate(rows)]).astype(np.float64)
    mx = x.max(axis=1, keepdims=True)
    want_lp = x - mx - np.log(np.exp(x - mx).sum(axis=1, keepdims=True))
    assert np.abs(lp - want_lp).max() / (1 + np.abs(want_lp).max()) < 1e-5
    m.close()


@pytest.mark.parametrize("quantized", [False, True])
def test_first_block_fc1_fp16_matches_oracle_and_reference(O, R, tmp_path, cuda, quantized):
    """esm.first_block_fc1_fp16 (model.cpp:1031-1033) on the device: layer 0's
    fc1 input rounded to fp16 (and, per tensor, its absmax taken after the
    rounding) against the oracle and the compiled reference loading the same
    GGUF."""
    from esm_b200 import Model, synth

    m = synth.random_model(TINY, seed=41)
    if quantized:
        stats = m.calibrate(synth.residue_ids([40, 60, 90], seed=42))
        m.apply_smoothquant(stats, 0.5)
        m.quantize_weights()
    m.set_first_block_fc1_fp16(True)
    gg = tmp_path / "fc1fp16.gguf"
    m.save_to_gguf(gg)
    dev = Model.load(gg)
    assert dev.config.first_block_fc1_fp16
    seqs, ids, cu = _batch([40, 3, 130, 250], 43)
    got = dev.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(dev, ids, cu)
    O.ref_force_isa("avx512vnni")
    try:
        rw = O.RefModel(gg).forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    if quantized:
        for w in (want, rw):
            np.testing.assert_allclose(got, w, rtol=1e-3, atol=W8A8_ATOL)
            _pearson_each(got, w, cu)
    else:
        _close(got, want)
        _close(got, rw)
    dev.close()
    m.close()


@pytest.mark.parametrize("which", ["fp32", "q8"])
def test_bf16_attention_forward_matches_oracle(which, tiny_fp32, tiny_q8, O, monkeypatch):
    """ESM_AMX_ATTENTION=on through the whole forward: Q and K rounded to bf16
    after the scale and RoPE, as the reference's AttentionVarlenAvx512Bf16
    does, against the oracle's forward with the same switch."""
    m = tiny_fp32 if which == "fp32" else tiny_q8
    seqs, ids, cu = _batch([40, 3, 130, 300], 52)
    off = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    monkeypatch.setenv("ESM_AMX_ATTENTION", "on")
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    want = O.forward_packed(m, ids, cu)
    if which == "fp32":
        _close(got, want)
        assert np.abs(got - off).max() > 1e-5
    else:
        np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)
        _pearson_each(got, want, cu)


def test_streaming_scheduler_matches_forward_scheduled(tiny_fp32):
    """esm_b200.streaming over two replicas (both on device 0 here): every
    request's logits equal its rows of one forward_scheduled over all the
    sequences (FP32: batch mates change nothing beyond rounding)."""
    from esm_b200 import Model, synth
    from esm_b200.streaming import StreamingScheduler

    other = Model(tiny_fp32.config, tiny_fp32.embed, tiny_fp32.layers, tiny_fp32.head, device=0)
    seqs = synth.residue_ids(synth.varlen_lengths(60, seed=81, mean=60, sd=40, lo=3, hi=300), seed=82)
    want = tiny_fp32.forward_scheduled(seqs)
    with StreamingScheduler([tiny_fp32, other], max_tokens=1500, max_wait_ms=2) as s:
        futs = s.submit_many(seqs)
        got = [f.result(timeout=60) for f in futs]
    for g, w in zip(got, want):
        assert g.shape == w.shape
        _close(g, w, tol=1e-5)
    other.close()
