"""Zero-shot masked-marginal scoring of deep-mutational-scan assays, with the
semantics of the reference's esm_cpp.eval.proteingym
(python/esm_cpp/eval/proteingym.py:1-162) on this package's device head.

For an assay (a wild type and variants of the same length):
  - every position p where some variant differs from the wild type is masked
    in one copy of the wild type; the copies run once through the scheduled
    forward;
  - a variant scores  sum over its substitutions (p, wt_aa, mut_aa) of
    log P(mut_aa | p masked) - log P(wt_aa | p masked);
  - Spearman(scores, experimental fitness) is the assay's metric.

The reference brings every copy's full [L, V] logits back to the host and
takes one row of each.  Here Model.masked_marginals runs the LM head on
those rows alone and returns their log-softmax, [P, V] for P masked
positions: the host reads P*V floats instead of P*L*V.
"""
from __future__ import annotations

import csv
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable

import numpy as np

# The 33-token ESM-2 vocabulary in id order (tokenizer.cpp:12-17): the rows
# of the embedding and the columns of the logits.
ESM2_VOCAB = (
    "<cls>", "<pad>", "<eos>", "<unk>",
    "L", "A", "G", "V", "S", "E", "R", "T", "I", "D", "P", "K", "Q", "N",
    "F", "Y", "M", "H", "W", "C", "X", "B", "U", "Z", "O", ".", "-",
    "<null_1>", "<mask>",
)


class ResidueTokenizer:
    """The part of esm::Tokenizer (tokenizer.h:24-66) that scoring needs:
    encode() of a plain residue string (ASCII whitespace dropped, one token
    per vocabulary character, <cls> ... <eos> around it), token_to_id() and
    mask_id.  Special-token text and unknown characters, which the reference
    tokenizer matches greedily or collapses to <unk>, raise ValueError here;
    any object with these three members (the reference's own Tokenizer
    included) can be passed to score_assay instead."""

    cls_id, pad_id, eos_id, unk_id, mask_id = 0, 1, 2, 3, 32

    def __init__(self):
        self._id = {tok: i for i, tok in enumerate(ESM2_VOCAB)}

    def token_to_id(self, token: str) -> int:
        """Exact token string -> id, <unk> for anything else (tokenizer.h:55-56)."""
        return self._id.get(token, self.unk_id)

    def encode(self, sequence: str) -> list[int]:
        out = [self.cls_id]
        for ch in sequence:
            if ch in " \t\n\r\v\f":
                continue
            i = self._id.get(ch)
            if i is None or len(ESM2_VOCAB[i]) != 1:
                raise ValueError(f"{ch!r} is not a residue character of the ESM-2 vocabulary")
            out.append(i)
        out.append(self.eos_id)
        return out


@dataclass(frozen=True)
class Variant:
    """One DMS variant of the wild type and its experimental fitness."""
    sequence: str
    fitness: float

    def diffs_from(self, wt: str) -> list[tuple[int, str, str]]:
        """(position, wild-type residue, variant residue) where they differ."""
        if len(self.sequence) != len(wt):
            raise ValueError("variant and wt must have equal length")
        return [(i, a, b) for i, (a, b) in enumerate(zip(wt, self.sequence)) if a != b]


def masked_log_probs(model, wt_ids, positions, imbalance_threshold: float = 1.2,
                     max_batch_size: int = 256) -> np.ndarray:
    """[len(positions), V]: log-softmax of the logits at model row p + 1
    (after <cls>) of the wild type with residue p masked, one masked copy
    per position (eval/proteingym.py:75-88)."""
    wt_ids = np.ascontiguousarray(wt_ids, np.int32)
    pos = [int(p) for p in positions]
    copies = []
    for p in pos:
        x = wt_ids.copy()
        x[p + 1] = ResidueTokenizer.mask_id
        copies.append(x)
    rows = np.array([p + 1 for p in pos], np.int32)
    return model.masked_marginals(copies, rows, imbalance_threshold=imbalance_threshold,
                                  max_batch_size=max_batch_size)


def score_assay(model, tokenizer, wt_sequence: str, variants: Iterable[Variant],
                imbalance_threshold: float = 1.2,
                max_batch_size: int = 256) -> tuple[list[float], list[float]]:
    """(scores, fitnesses) aligned by variant (eval/proteingym.py:53-101)."""
    variants = list(variants)
    if not variants:
        return [], []
    diffs = [v.diffs_from(wt_sequence) for v in variants]
    positions = sorted({p for d in diffs for p, _, _ in d})
    lp = {}
    if positions:
        table = masked_log_probs(model, tokenizer.encode(wt_sequence), positions,
                                 imbalance_threshold, max_batch_size)
        lp = {p: table[i] for i, p in enumerate(positions)}
    scores = []
    for d in diffs:
        s = 0.0
        for p, wt_aa, mut_aa in d:
            row = lp[p]
            s += float(row[tokenizer.token_to_id(mut_aa)]) - float(row[tokenizer.token_to_id(wt_aa)])
        scores.append(s)
    return scores, [v.fitness for v in variants]


def rankdata(xs) -> np.ndarray:
    """1-based ranks, ties sharing their average rank (eval/proteingym.py:121-134)."""
    x = np.asarray(xs, np.float64)
    order = np.argsort(x, kind="stable")
    ranks = np.empty(x.size, np.float64)
    i = 0
    while i < x.size:
        j = i
        while j + 1 < x.size and x[order[j + 1]] == x[order[i]]:
            j += 1
        ranks[order[i:j + 1]] = (i + j + 2) / 2.0
        i = j + 1
    return ranks


def spearman(xs, ys) -> float:
    """Spearman rank correlation; 0.0 for fewer than two points or a
    constant input (eval/proteingym.py:104-118)."""
    if len(xs) < 2:
        return 0.0
    rx, ry = rankdata(xs), rankdata(ys)
    dx, dy = rx - rx.mean(), ry - ry.mean()
    nx, ny = math.sqrt(float((dx * dx).sum())), math.sqrt(float((dy * dy).sum()))
    if nx == 0.0 or ny == 0.0:
        return 0.0
    return float((dx * dy).sum()) / (nx * ny)


def load_assay_csv(path) -> tuple[str, list[Variant]]:
    """A ProteinGym-format assay CSV (eval/proteingym.py:137-162): columns
    mutated_sequence and DMS_score; the wild type is the row whose `mutant`
    is WT (else the first row); rows without a numeric DMS_score are
    skipped."""
    rows = list(csv.DictReader(Path(path).open("r")))
    if not rows:
        raise ValueError(f"empty assay file {path}")
    is_wt = [r.get("mutant", "").upper() == "WT" for r in rows]
    wt = rows[is_wt.index(True) if any(is_wt) else 0]["mutated_sequence"]
    variants = []
    for r, w in zip(rows, is_wt):
        if w:
            continue
        try:
            fitness = float(r["DMS_score"])
        except (KeyError, ValueError):
            continue
        variants.append(Variant(sequence=r["mutated_sequence"], fitness=fitness))
    return wt, variants
