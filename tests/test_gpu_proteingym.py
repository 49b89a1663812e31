"""The masked-marginal head on the GPU (esmcu_model_masked_marginals):
LM head on the scored rows only + device log-softmax.

Gates:
  - against log-softmax of the same device's full forward_scheduled logits
    (the head is row-wise FP32, so only GEMM tiling differs): 1e-5;
  - against the oracle and the compiled reference: the whole-forward gates
    of test_gpu_model.py (FP32 1e-4 * (1 + |ref|); W8A8 |d| <= 5e-2);
  - score_assay against the reference's own loop (eval/proteingym.py:63-101)
    on the compiled reference, and the reference's test cases
    (tests/python/test_proteingym.py:63-109).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TINY = dict(num_hidden_layers=2, hidden_size=128, num_attention_heads=2, head_dim=64,
            intermediate_size=512)
W8A8_ATOL = 5e-2


def _rel(got, want):
    return float((np.abs(got - want) / (1.0 + np.abs(want))).max())


def _log_softmax(rows):
    x = rows.astype(np.float64)
    m = x.max(axis=1, keepdims=True)
    return (x - m - np.log(np.exp(x - m).sum(axis=1, keepdims=True))).astype(np.float32)


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


def _seqs_rows(lens, seed):
    from esm_b200 import synth

    seqs = synth.residue_ids(lens, seed=seed)
    rng = np.random.default_rng(seed)
    rows = np.array([rng.integers(0, len(s)) for s in seqs], np.int32)
    return seqs, rows


@pytest.mark.parametrize("which", ["fp32", "q8"])
def test_matches_full_logits_and_oracle(which, tiny_fp32, tiny_q8, O):
    m = tiny_fp32 if which == "fp32" else tiny_q8
    seqs, rows = _seqs_rows([1, 17, 130, 250, 64, 3, 200, 90], 21)
    got = m.masked_marginals(seqs, rows, max_batch_size=4)
    assert got.shape == (len(seqs), 33) and np.isfinite(got).all()
    full = m.forward_scheduled(seqs, max_batch_size=4)
    want_dev = _log_softmax(np.stack([full[i][r] for i, r in enumerate(rows)]))
    assert _rel(got, want_dev) < 1e-5
    # Probabilities sum to one.
    np.testing.assert_allclose(np.exp(got.astype(np.float64)).sum(axis=1), 1.0, atol=1e-5)
    want = O.masked_marginals(m, seqs, rows, 1.2, 4)
    if which == "fp32":
        assert _rel(got, want) < 1e-4
    else:
        np.testing.assert_allclose(got, want, rtol=1e-3, atol=W8A8_ATOL)


def test_score_assay_matches_reference_loop(tiny_fp32, O, R, tmp_path):
    """score_assay on the device head against the reference's algorithm on
    the reference's own Model::ForwardScheduled (compiled, same weights)."""
    from esm_b200.proteingym import ResidueTokenizer, Variant, score_assay, spearman

    p = tmp_path / "tiny_pg.safetensors"
    tiny_fp32.save_to_safetensors(p)
    ref = O.RefModel(p)
    tok = ResidueTokenizer()
    rng = np.random.default_rng(5)
    alphabet = "LAGVSERTIDPKQNFYMHWC"
    wt = "".join(rng.choice(list(alphabet), 120))
    variants = []
    for k in range(40):
        s = list(wt)
        for pos in rng.choice(len(wt), int(rng.integers(1, 4)), replace=False):
            s[pos] = rng.choice([a for a in alphabet if a != wt[pos]])
        variants.append(Variant("".join(s), float(rng.standard_normal())))
    variants.append(Variant(wt, 0.0))
    scores, fit = score_assay(tiny_fp32, tok, wt, variants)
    # The reference's loop (eval/proteingym.py:63-101) on its own forward.
    wt_ids = np.array(tok.encode(wt), np.int32)
    pos = sorted({q for v in variants for q, _, _ in v.diffs_from(wt)})
    copies = []
    for q in pos:
        x = wt_ids.copy()
        x[q + 1] = tok.mask_id
        copies.append(x)
    row_at = {q: lg[q + 1] for q, lg in zip(pos, ref.forward_scheduled(copies))}
    want = [sum(O.log_softmax_at(row_at[q], tok.token_to_id(b)) -
                O.log_softmax_at(row_at[q], tok.token_to_id(a)) for q, a, b in v.diffs_from(wt))
            for v in variants]
    np.testing.assert_allclose(scores, want, rtol=0, atol=2e-4)
    assert scores[-1] == 0.0
    assert abs(spearman(scores, fit) - spearman(want, fit)) < 0.05


def test_reference_cases(tiny_q8):
    """tests/python/test_proteingym.py:63-109 on a W8A8 model."""
    from esm_b200.proteingym import ResidueTokenizer, Variant, score_assay, spearman

    tok = ResidueTokenizer()
    wt = "MKTGVAQRLELDSPMVLQ"
    assert score_assay(tiny_q8, tok, wt, [Variant(wt, 1.0)]) == ([0.0], [1.0])
    assert wt[6] == "Q"
    (s,), _ = score_assay(tiny_q8, tok, wt, [Variant(wt[:6] + "A" + wt[7:], 0.5)])
    assert s != 0.0 and s == s
    # The single-substitution score is log P(A | masked 6) - log P(Q | masked 6).
    x = np.array(tok.encode(wt), np.int32)
    x[7] = tok.mask_id
    lp = tiny_q8.masked_marginals([x], np.array([7], np.int32))[0]
    assert s == float(lp[tok.token_to_id("A")]) - float(lp[tok.token_to_id("Q")])
    wt = "MKTGVAQRLELDSPMVLQKR"
    vs = [Variant(wt[:5] + "A" + wt[6:], 0.8), Variant(wt[:5] + "L" + wt[6:], 0.6),
          Variant(wt[:7] + "K" + wt[8:], 0.3), Variant(wt[:7] + "E" + wt[8:], 0.1),
          Variant(wt[:10] + "A" + wt[11:], 0.5), Variant(wt[:10] + "D" + wt[11:], 0.0)]
    scores, fit = score_assay(tiny_q8, tok, wt, vs)
    assert len(scores) == 6 and all(v == v for v in scores)
    assert -1.0 <= spearman(scores, fit) <= 1.0


def test_dms_shape_against_full_forward(tiny_fp32, O):
    """A 400-residue wild type masked at every position (402-token copies,
    the deep-mutational-scan shape): the head matches the full forward's
    rows at full size, and the oracle on a few positions."""
    from esm_b200 import synth

    wt = synth.dms_sequences(seed=7, length=400)[0]
    copies, rows = [], []
    for p in range(400):
        x = wt.copy()
        x[p + 1] = 32
        copies.append(x)
        rows.append(p + 1)
    rows = np.array(rows, np.int32)
    got = tiny_fp32.masked_marginals(copies, rows)
    full = tiny_fp32.forward_scheduled(copies)
    assert _rel(got, _log_softmax(np.stack([full[i][r] for i, r in enumerate(rows)]))) < 1e-5
    pick = [0, 57, 199, 399]
    want = O.masked_marginals(tiny_fp32, [copies[i] for i in pick], rows[pick])
    assert _rel(got[pick], want) < 1e-4


def test_rejects_rows_out_of_range(tiny_fp32):
    from esm_b200 import EsmCudaError, _lib, synth

    seqs = synth.residue_ids([10, 20], seed=1)
    n0, n1 = len(seqs[0]), len(seqs[1])
    for bad in ([n0, 0], [0, -1], [0, n1]):
        with pytest.raises(EsmCudaError) as ei:
            tiny_fp32.masked_marginals(seqs, np.array(bad, np.int32))
        assert _lib.STATUS[ei.value.code] == "OUT_OF_RANGE"
    with pytest.raises(ValueError):
        tiny_fp32.masked_marginals(seqs, np.array([0], np.int32))
    assert tiny_fp32.masked_marginals([], np.zeros(0, np.int32)).shape == (0, 33)
    # The model stays usable.
    assert np.isfinite(tiny_fp32.masked_marginals(seqs, np.array([n0 - 1, n1 - 1], np.int32))).all()
