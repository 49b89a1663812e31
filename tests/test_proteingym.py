"""Masked-marginal scoring host logic (esm_b200.proteingym) -- CPU only.

Mirrors the reference's tests/python/test_proteingym.py (Spearman cases,
zero-diff and single-substitution scores, a mini assay) with the model's
device head replaced by the oracle, and pins the oracle's masked marginals
against the reference compiled in oracle/_ref.
"""
import numpy as np
import pytest

from pathlib import Path

GOLD = Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------- Spearman
def test_spearman_reference_cases():
    """tests/python/test_proteingym.py:37-60."""
    from esm_b200.proteingym import spearman

    assert abs(spearman([1, 2, 3, 4, 5], [10, 20, 30, 40, 50]) - 1.0) < 1e-9
    assert abs(spearman([1, 2, 3, 4, 5], [50, 40, 30, 20, 10]) + 1.0) < 1e-9
    assert -1.0 <= spearman([1.0, 1.0, 2.0, 3.0], [4.0, 5.0, 6.0, 7.0]) <= 1.0
    assert spearman([1.0, 1.0, 1.0], [1.0, 2.0, 3.0]) == 0.0
    assert spearman([1.0], [2.0]) == 0.0


def test_rankdata_and_spearman_match_scipy():
    from scipy import stats

    from esm_b200.proteingym import rankdata, spearman

    rng = np.random.default_rng(0)
    for n in (2, 7, 100):
        x = rng.integers(0, 5, n).astype(float)  # many ties
        y = rng.standard_normal(n)
        assert np.array_equal(rankdata(x), stats.rankdata(x))
        want = stats.spearmanr(x, y).statistic
        if np.isnan(want):
            assert spearman(list(x), list(y)) == 0.0
        else:
            assert abs(spearman(list(x), list(y)) - want) < 1e-12


# ------------------------------------------------------------ tokenizer
def test_residue_tokenizer():
    from esm_b200 import MASK_ID
    from esm_b200.proteingym import ESM2_VOCAB, ResidueTokenizer

    t = ResidueTokenizer()
    assert len(ESM2_VOCAB) == 33 and ESM2_VOCAB[MASK_ID] == "<mask>"
    # tokenizer.cpp:12-17: L=4 A=5 ... M=20 K=15 T=11.
    assert t.encode("MKT") == [0, 20, 15, 11, 2]
    assert t.encode(" M K\nT\t") == [0, 20, 15, 11, 2]
    assert t.token_to_id("Q") == 16 and t.token_to_id("<mask>") == 32
    assert t.token_to_id("J") == 3 and t.mask_id == 32
    for bad in ("MJK", "M<mask>K"):
        with pytest.raises(ValueError):
            t.encode(bad)


def test_variant_diffs():
    from esm_b200.proteingym import Variant

    assert Variant("MKTA", 0.0).diffs_from("MKTG") == [(3, "G", "A")]
    assert Variant("MKTG", 0.0).diffs_from("MKTG") == []
    with pytest.raises(ValueError):
        Variant("MKT", 0.0).diffs_from("MKTG")


def test_load_assay_csv(tmp_path):
    from esm_b200.proteingym import load_assay_csv

    p = tmp_path / "a.csv"
    p.write_text("mutant,mutated_sequence,DMS_score\n"
                 "K2A,MATG,0.5\nWT,MKTG,1.0\nT3L,MKLG,nan-ish\nG4V,MKTV,-0.25\n")
    wt, vs = load_assay_csv(p)
    assert wt == "MKTG"
    assert [(v.sequence, v.fitness) for v in vs] == [("MATG", 0.5), ("MKTV", -0.25)]
    q = tmp_path / "b.csv"
    q.write_text("mutated_sequence,DMS_score\nMKTG,1.0\nMKTA,0.5\n")
    wt, vs = load_assay_csv(q)
    assert wt == "MKTG" and [v.sequence for v in vs] == ["MKTG", "MKTA"]
    e = tmp_path / "c.csv"
    e.write_text("mutated_sequence,DMS_score\n")
    with pytest.raises(ValueError):
        load_assay_csv(e)


# ----------------------------------------------------- scoring host logic
class _OracleHead:
    """A model whose masked_marginals is the oracle's (CPU)."""

    def __init__(self, O, model):
        self.O, self.model, self.calls = O, model, []

    def masked_marginals(self, seqs, rows, imbalance_threshold=1.2, max_batch_size=256):
        self.calls.append(([s.copy() for s in seqs], np.asarray(rows).copy()))
        return self.O.masked_marginals(self.model, seqs, rows, imbalance_threshold, max_batch_size)


@pytest.fixture(scope="module")
def golden_fp32(tmp_path_factory):
    from esm_b200 import Model

    M = np.load(GOLD / "model_golden.npz")
    p = tmp_path_factory.mktemp("pg") / "m.safetensors"
    p.write_bytes(M["safetensors"].tobytes())
    return Model.load(p), p


def _literal_scores(O, model, tok, wt, variants):
    """The reference's loop written out (eval/proteingym.py:63-101): one
    masked wild type per mutated position, one forward per copy."""
    wt_ids = np.array(tok.encode(wt), np.int32)
    out = []
    for v in variants:
        s = 0.0
        for p, a, b in v.diffs_from(wt):
            x = wt_ids.copy()
            x[p + 1] = tok.mask_id
            row = O.forward_packed(model, x, np.array([0, x.size], np.int32))[p + 1]
            s += O.log_softmax_at(row, tok.token_to_id(b)) - O.log_softmax_at(row, tok.token_to_id(a))
        out.append(s)
    return out


def test_score_assay_host_logic(O, golden_fp32):
    from esm_b200.proteingym import ResidueTokenizer, Variant, score_assay, spearman

    model, _ = golden_fp32
    tok = ResidueTokenizer()
    wt = "MKTGVAQRLELDSPMVLQKR"
    variants = [Variant(wt[:5] + "A" + wt[6:], 0.8), Variant(wt[:5] + "L" + wt[6:], 0.6),
                Variant(wt[:7] + "K" + wt[8:], 0.3), Variant(wt[:7] + "E" + wt[8:], 0.1),
                Variant(wt[:10] + "A" + wt[11:], 0.5), Variant(wt[:3] + "AA" + wt[5:], 0.0),
                Variant(wt, 1.0)]
    head = _OracleHead(O, model)
    scores, fit = score_assay(head, tok, wt, variants)
    assert fit == [v.fitness for v in variants]
    # One masked copy per distinct position, in sorted order, scored at p + 1.
    (seqs, rows), = head.calls
    assert rows.tolist() == [p + 1 for p in (3, 4, 5, 7, 10)]
    for s, p in zip(seqs, (3, 4, 5, 7, 10)):
        assert s[p + 1] == tok.mask_id and s.size == len(wt) + 2
    assert scores[-1] == 0.0  # tests/python/test_proteingym.py:63-70
    want = _literal_scores(O, model, tok, wt, variants)
    np.testing.assert_allclose(scores, want, rtol=0, atol=1e-5)
    assert -1.0 <= spearman(scores, fit) <= 1.0
    assert score_assay(head, tok, wt, []) == ([], [])


def test_oracle_masked_marginals_match_reference(O, R, golden_fp32):
    """The oracle's scheduled forward + log-softmax against the reference's
    Model::ForwardScheduled (compiled) + the same formula."""
    model, path = golden_fp32
    from esm_b200 import synth

    seqs = synth.residue_ids([30, 7, 64, 30], seed=4)
    rows = np.array([5, 0, 63, 29], np.int32)
    got = O.masked_marginals(model, seqs, rows)
    ref_logits = O.RefModel(path).forward_scheduled(seqs)
    want = np.array([[O.log_softmax_at(ref_logits[i][r], t) for t in range(33)]
                     for i, r in enumerate(rows)], np.float32)
    assert (np.abs(got - want) / (1 + np.abs(want))).max() < 1e-4
