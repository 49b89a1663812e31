"""Host-side logic on the CPU: weight files (safetensors, GGUF Q8_ESM) read
and written in the reference's formats, the load-time quantisation, and
SmoothQuant migration."""
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
TINY = dict(num_hidden_layers=2, hidden_size=64, num_attention_heads=1, head_dim=64,
            intermediate_size=256)


def test_quantize_weight_bitexact_vs_oracle_and_reference(O, R):
    from esm_b200.prep import quantize_weight

    rng = np.random.default_rng(0)
    for N, K in [(1, 16), (64, 80), (1280, 1280)]:
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        W[0] = 0.0
        q, s = quantize_weight(W)
        qo, so = O.quantize_weights(W)
        assert np.array_equal(q, qo) and np.array_equal(s, so)
        qr = np.zeros((N, K), np.int8)
        sr = np.zeros(N, np.float32)
        R.ref_quantize_weights(W.ctypes.data, N, K, qr.ctypes.data, sr.ctypes.data)
        assert np.array_equal(q, qr) and np.array_equal(s, sr)


def test_safetensors_round_trip(tmp_path):
    from esm_b200 import Model, synth

    m = synth.random_model(TINY, seed=1)
    p = tmp_path / "m.safetensors"
    m.save_to_safetensors(p)
    m2 = Model.load(p)
    assert m2.config.num_hidden_layers == 2 and m2.config.head_dim == 64
    assert m2.config.num_attention_heads == 1 and m2.config.intermediate_size == 256
    assert np.array_equal(m2.embed, m.embed)
    for a, b in zip(m.layers, m2.layers):
        for k in a:
            assert np.array_equal(a[k], b[k])


def test_gguf_round_trip_quantized(tmp_path):
    from esm_b200 import Model, synth

    m = synth.random_model(TINY, seed=2)
    m.quantize_weights()
    p = tmp_path / "m.gguf"
    m.save_to_gguf(p)
    m2 = Model.load(p)
    assert m2.config.weights_quantized
    for a, b in zip(m.layers, m2.layers):
        for n in ("q", "k", "v", "out", "fc1", "fc2"):
            assert np.array_equal(a[n + "_wq"], b[n + "_wq"])
            assert np.array_equal(a[n + "_ws"], b[n + "_ws"])
            assert np.array_equal(a[n + "_b"], b[n + "_b"])
    for k in m.head:
        assert np.array_equal(m.head[k], m2.head[k])


def test_reference_reads_our_gguf_and_we_read_its(O, R, tmp_path):
    """Both engines consume one artefact: the reference loads the GGUF this
    package writes, and this package loads the one the reference writes."""
    from esm_b200 import Model, synth

    m = synth.random_model(TINY, seed=3)
    m.quantize_weights()
    p = tmp_path / "ours.gguf"
    m.save_to_gguf(p)
    ref = O.RefModel(p)
    assert (ref.layers, ref.d, ref.heads, ref.dh, ref.ffn, ref.quantized) == (2, 64, 1, 64, 256, 1)
    p2 = tmp_path / "theirs.gguf"
    ref.save_gguf(p2)
    m2 = Model.load(p2)
    for a, b in zip(m.layers, m2.layers):
        assert np.array_equal(a["fc1_wq"], b["fc1_wq"]) and np.array_equal(a["fc1_ws"], b["fc1_ws"])


def test_golden_gguf_loads():
    from esm_b200 import Model

    M = np.load(ROOT / "tests" / "golden" / "model_golden.npz")
    import tempfile

    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "g.gguf"
        p.write_bytes(M["gguf_q8"].tobytes())
        m = Model.load(p)
    assert m.config.weights_quantized and m.config.hidden_size == 64
    assert m.layers[0]["q_wq"].dtype == np.int8 and m.layers[0]["q_wq"].shape == (64, 64)


def test_smoothquant_scales_follow_reference_formula():
    from esm_b200.prep import smoothquant_scales

    s = smoothquant_scales(np.array([4.0, 0.0, 1e9, 1.0], np.float32),
                           np.array([1.0, 1.0, 1e-9, 0.0], np.float32), 0.5)
    assert s[0] == 2.0 and s[1] == 1.0 and s[2] == np.float32(1e3) and s[3] == 1.0


def test_smoothquant_preserves_fp32_function(O):
    """tests/cpp/test_smoothquant.cpp:76-125: migration is an identity of the
    FP32 forward (to rounding): LN gamma/beta /= s, W[:, k] *= s[k]."""
    from esm_b200 import synth

    m = synth.random_model(TINY, seed=4)
    seqs = synth.residue_ids([20, 33], seed=5)
    ids, cu = synth.pack(seqs)
    before = O.forward_packed(m, ids, cu)
    stats = {f"layer{i}.{s}": 3.0 for i in range(2)
             for s in ("attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu")}
    m.apply_smoothquant(stats, 0.5)
    after = O.forward_packed(m, ids, cu)
    assert np.abs(after - before).max() < 1e-4


def test_apply_smoothquant_refuses_quantized():
    from esm_b200 import synth

    m = synth.random_model(TINY, seed=6)
    m.quantize_weights()
    with pytest.raises(RuntimeError):
        m.apply_smoothquant({}, 0.5)


def test_synthetic_workloads_have_baseline_shapes():
    from esm_b200 import synth

    lens = synth.varlen_lengths(256, seed=1000)
    assert lens.min() >= 90 and lens.max() <= 250 and abs(lens.mean() - 120) < 6
    seqs = synth.residue_ids(lens, seed=2000)
    assert all(s[0] == 0 and s[-1] == 2 and s[1:-1].min() >= 4 and s[1:-1].max() <= 23 for s in seqs)
    dms = synth.dms_sequences(0, length=10)
    assert len(dms) == 1 + 19 * 10 and all(len(s) == 12 for s in dms)


def test_isa_queries():
    """esm_cpp.current_isa / host_isa (_core.cpp:83-89): this engine has one
    target."""
    import esm_b200

    assert esm_b200.current_isa() == esm_b200.host_isa() == "sm_100a"


def test_host_smoothquant_migration_matches_reference_bits(O, R, tmp_path):
    """prep.migrate_smoothquant (the host path of Model.apply_smoothquant)
    against the compiled reference's ApplySmoothQuant on the same FP32
    weights and statistics: every migrated tensor bit-identical."""
    from esm_b200 import Model, synth

    arch = dict(num_hidden_layers=2, hidden_size=320, num_attention_heads=20, head_dim=16,
                intermediate_size=1280)
    m = synth.random_model(arch, seed=23)
    m.save_to_safetensors(tmp_path / "w.safetensors")
    rng = np.random.default_rng(24)
    sites = ("attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu")
    st = (rng.random(8) * 20 + 0.1).astype(np.float32)
    st[1] = 0.0  # a site with no statistic: s = 1
    stats = {f"layer{i}.{sites[j]}": float(st[i * 4 + j]) for i in range(2) for j in range(4)}
    ref = O.RefModel(tmp_path / "w.safetensors")
    ref.apply_smoothquant(st, 0.5)
    ref.save_gguf(tmp_path / "m.gguf")
    want = Model.load_from_gguf(tmp_path / "m.gguf")
    m.apply_smoothquant(stats, 0.5)
    for i in range(2):
        for name, a in m.layers[i].items():
            assert np.array_equal(a.view(np.uint32), want.layers[i][name].view(np.uint32)), (i, name)
