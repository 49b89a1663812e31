"""On-device weight preparation against the reference compiled from its own
sources: the SmoothQuant migration (esmcu_model_apply_smoothquant,
smoothquant.cpp:100-185) and per-channel quantisation
(esmcu_model_quantize_weights, pack.cpp:149-177) of a replica in HBM give the
reference's weights bit for bit from the same statistics; the calibration
observer (esmcu_observer fed by the GPU forward) gives the reference's
ForwardWithObserver percentiles to the FP32 class -- the reservoir keeps the
same positions, and the values there are the two engines' FP32 activations.
"""
import tempfile
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ARCH = dict(num_hidden_layers=2, hidden_size=1280, num_attention_heads=20, head_dim=64,
            intermediate_size=5120)
SITES = ("attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu")
FP32_NAMES = ("attn_ln_w", "attn_ln_b", "ffn_ln_w", "ffn_ln_b", "q_w", "k_w", "v_w", "out_w",
              "fc1_w", "fc2_w", "q_b", "k_b", "v_b", "out_b", "fc1_b", "fc2_b")


@pytest.fixture(scope="module")
def prep(cuda, O, R):
    from esm_b200 import synth

    td = tempfile.TemporaryDirectory()
    p = Path(td.name)
    m = synth.random_model(ARCH, seed=17)
    m.save_to_safetensors(p / "w.safetensors")
    calib = synth.residue_ids(synth.varlen_lengths(6, seed=18), seed=19)
    yield m, calib, p
    m.close()
    td.cleanup()


def test_observer_stats_match_reference(prep, O, record):
    m, calib, p = prep
    if m.config.weights_quantized:
        pytest.skip("needs the FP32 model")
    got = m.calibrate(calib, 99.9)
    want = O.RefModel(p / "w.safetensors").observe(calib, 99.9)
    n = m.config.num_hidden_layers
    worst = 0.0
    for i in range(n):
        for j, site in enumerate(SITES):
            g, w = got[f"layer{i}.{site}"], float(want[i * 4 + j])
            worst = max(worst, abs(g - w) / max(abs(w), 1e-30))
    record("observer_stats_vs_reference", sites=4 * n, max_rel_diff=worst)
    assert worst <= 1e-4, worst


def test_device_smoothquant_and_quantize_match_reference_bits(prep, O, record):
    from esm_b200 import Model

    m, calib, p = prep
    stats = m.calibrate(calib, 99.9)
    n = m.config.num_hidden_layers
    st = np.array([stats[f"layer{i}.{SITES[j]}"] for i in range(n) for j in range(4)], np.float32)
    # Reference: the same FP32 weights, the same statistics.
    ref = O.RefModel(p / "w.safetensors")
    ref.apply_smoothquant(st, 0.5)
    ref.save_gguf(p / "ref_migrated.gguf")
    ref.quantize()
    ref.save_gguf(p / "ref_q8.gguf")
    # Ours, in HBM.
    host = Model.load_from_safetensors(p / "w.safetensors")  # the numpy restatement, for the record
    host.apply_smoothquant(stats, 0.5)
    m.apply_smoothquant(stats, 0.5, on_device=True)
    rm = Model.load_from_gguf(p / "ref_migrated.gguf")
    host_same = True
    for i in range(n):
        for name in FP32_NAMES:
            a, b = m.layers[i][name], rm.layers[i][name]
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (i, name)
            host_same &= bool(np.array_equal(host.layers[i][name], b))
    m.quantize_weights(on_device=True)
    rq = Model.load_from_gguf(p / "ref_q8.gguf")
    for i in range(n):
        for ln in ("q", "k", "v", "out", "fc1", "fc2"):
            assert np.array_equal(m.layers[i][ln + "_wq"], rq.layers[i][ln + "_wq"]), (i, ln)
            assert np.array_equal(m.layers[i][ln + "_ws"].view(np.uint32),
                                  rq.layers[i][ln + "_ws"].view(np.uint32)), (i, ln)
    record("device_smoothquant_quantize", layers=n, bit_exact=True, host_path_bit_exact=host_same)
    assert host_same  # the host restatement (prep.py) gives the same bits
    # The replica in HBM is the quantised model: a forward runs on it as is.
    seqs = calib[:3]
    ids = np.concatenate(seqs).astype(np.int32)
    cu = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.int32)
    out = m.forward_packed(ids, cu, out=np.empty((ids.size, 33), np.float32))
    assert np.isfinite(out).all()
