"""ESM-2 650M (BASELINE config 3 architecture, random-init weights) against
the reference compiled from its own sources, one packed group of 8
sequences (residues ~ N(120,30) clipped to [90,250]):

  FP32: logits within 1e-4 * (1 + |ref|), per-sequence Pearson >= 0.99999 --
        every FP32 kernel (LN, 3xTF32 tensor-core attention, RoPE, GELU,
        FP32 GEMMs) agrees with the reference's AVX-512 path.
  W8A8: the reference calibrates nothing here; both engines load one GGUF
        (this package's calibration + SmoothQuant + Quantize).  Logit
        agreement must be at least the reference's agreement with itself
        across its VNNI and default (AMX on Sapphire Rapids) paths, minus a
        small margin, and Pearson >= 0.998.
"""
import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pearson_min(a, b, cu):
    return min(np.corrcoef(a[cu[i]:cu[i + 1]].ravel(), b[cu[i]:cu[i + 1]].ravel())[0, 1]
               for i in range(len(cu) - 1))


@pytest.fixture(scope="module")
def setup(cuda, O, R):
    from esm_b200 import synth

    os.environ.setdefault("ESM_NUM_THREADS", str(os.cpu_count()))
    seqs = synth.residue_ids(synth.varlen_lengths(8, seed=5), seed=6)
    ids, cu = synth.pack(seqs)
    m = synth.random_model("esm2_650m", seed=0)
    td = tempfile.TemporaryDirectory()
    yield m, ids, cu, Path(td.name)
    m.close()
    td.cleanup()


def test_650m_fp32_matches_reference(setup, O):
    m, ids, cu, td = setup
    st = td / "w.safetensors"
    m.save_to_safetensors(st)
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    O.ref_force_isa("avx512vnni")
    try:
        want = O.RefModel(st).forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    assert (np.abs(got - want) / (1 + np.abs(want))).max() <= 1e-4
    assert _pearson_min(got, want, cu) >= 0.99999


def test_650m_w8a8_within_reference_isa_spread(setup, O):
    from esm_b200 import synth

    m, ids, cu, td = setup
    stats = m.calibrate(synth.residue_ids(synth.varlen_lengths(32, seed=1), seed=2), 99.9)
    m.apply_smoothquant(stats, 0.5)
    m.quantize_weights()
    got = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    p = td / "w.gguf"
    m.save_to_gguf(p)
    O.ref_force_isa("avx512vnni")
    try:
        vnni = O.RefModel(p).forward_packed(ids, cu)
    finally:
        O.ref_force_isa(None)
    default = O.RefModel(p).forward_packed(ids, cu)
    ours = _pearson_min(got, vnni, cu)
    spread = _pearson_min(vnni, default, cu)
    assert ours >= 0.998
    assert ours >= min(spread, 0.9995) - 5e-4, (ours, spread)
    assert np.abs(got - vnni).mean() <= 2 * max(np.abs(vnni - default).mean(), 0.01)
