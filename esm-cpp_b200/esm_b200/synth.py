"""Seeded synthetic inputs and random-init weights with the shapes of the
BASELINE configurations (no checkpoints or datasets exist on this box):

  esm2_8m / esm2_150m / esm2_650m / esm2_3b  ESM-2 architectures, weights
      N(0, 0.02), LayerNorm gamma = 1, beta = 0.
  varlen_lengths   residue counts ~ Normal(120, 30) clipped to [90, 250]
                   (config 3a) or uniform in [lo, hi] (config 0).
  residue_ids      ids uniform over 4..23 wrapped with CLS=0 / EOS=2.
  dms_sequences    a 400-residue wild type plus all 19*400 single-site
                   substitutions (config 4).
"""
from __future__ import annotations

import numpy as np

from .model import Config, Model

F32 = np.float32

ARCHS = {
    "esm2_8m": dict(num_hidden_layers=6, hidden_size=320, num_attention_heads=20, head_dim=16,
                    intermediate_size=1280),
    "esm2_35m": dict(num_hidden_layers=12, hidden_size=480, num_attention_heads=20, head_dim=24,
                     intermediate_size=1920),
    "esm2_150m": dict(num_hidden_layers=30, hidden_size=640, num_attention_heads=20, head_dim=32,
                      intermediate_size=2560),
    "esm2_650m": dict(num_hidden_layers=33, hidden_size=1280, num_attention_heads=20, head_dim=64,
                      intermediate_size=5120),
    "esm2_3b": dict(num_hidden_layers=36, hidden_size=2560, num_attention_heads=40, head_dim=64,
                    intermediate_size=10240),
}


def random_model(arch, seed: int = 0, device: int = 0, num_layers: int | None = None,
                 std: float = 0.02) -> Model:
    """Random-init FP32 model: Linear weights/biases and embeddings N(0, std)."""
    spec = dict(ARCHS[arch]) if isinstance(arch, str) else dict(arch)
    if num_layers is not None:
        spec["num_hidden_layers"] = num_layers
    cfg = Config(**spec)
    rng = np.random.default_rng(seed)
    d, f, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size

    def n(*shape):
        return (rng.standard_normal(shape, dtype=F32) * F32(std)).astype(F32)

    layers = []
    for _ in range(cfg.num_hidden_layers):
        layers.append({
            "attn_ln_w": np.ones(d, F32), "attn_ln_b": np.zeros(d, F32),
            "q_w": n(d, d), "q_b": n(d), "k_w": n(d, d), "k_b": n(d), "v_w": n(d, d), "v_b": n(d),
            "out_w": n(d, d), "out_b": n(d),
            "ffn_ln_w": np.ones(d, F32), "ffn_ln_b": np.zeros(d, F32),
            "fc1_w": n(f, d), "fc1_b": n(f), "fc2_w": n(d, f), "fc2_b": n(d),
        })
    head = {"final_ln_w": np.ones(d, F32), "final_ln_b": np.zeros(d, F32),
            "lm_dense_w": n(d, d), "lm_dense_b": n(d),
            "lm_ln_w": np.ones(d, F32), "lm_ln_b": np.zeros(d, F32), "lm_bias": n(V)}
    return Model(cfg, n(V, d), layers, head, device)


def varlen_lengths(n: int, seed: int, mean: float = 120.0, sd: float = 30.0, lo: int = 90,
                   hi: int = 250) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.rint(rng.normal(mean, sd, n)), lo, hi).astype(np.int32)


def uniform_lengths(n: int, seed: int, lo: int, hi: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, n).astype(np.int32)


def residue_ids(residue_lengths, seed: int, wrap: bool = True) -> list[np.ndarray]:
    """Residue ids uniform over 4..23, wrapped with CLS=0 / EOS=2."""
    rng = np.random.default_rng(seed)
    out = []
    for L in residue_lengths:
        r = rng.integers(4, 24, int(L)).astype(np.int32)
        out.append(np.concatenate([[0], r, [2]]).astype(np.int32) if wrap else r)
    return out


def dms_sequences(seed: int, length: int = 400) -> list[np.ndarray]:
    """Wild type + all single-site substitutions over the 20 ids 4..23."""
    rng = np.random.default_rng(seed)
    wt = rng.integers(4, 24, length).astype(np.int32)
    seqs = [np.concatenate([[0], wt, [2]]).astype(np.int32)]
    for p in range(length):
        for aa in range(4, 24):
            if aa == wt[p]:
                continue
            m = wt.copy()
            m[p] = aa
            seqs.append(np.concatenate([[0], m, [2]]).astype(np.int32))
    return seqs


def pack(seqs):
    lens = np.array([len(s) for s in seqs], np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return np.concatenate(seqs).astype(np.int32), cu


def quantized_model(arch="esm2_650m", seed: int = 0, device: int = 0, calib_seqs: int = 32,
                    alpha: float = 0.5, num_layers: int | None = None) -> Model:
    """Config 3 / 4 weights: random init -> seeded calibration on the GPU
    (percentile 99.9) -> SmoothQuant(alpha) -> per-channel int8, the last
    two on the replica in HBM (the same bits as the host path)."""
    m = random_model(arch, seed=seed, device=device, num_layers=num_layers)
    calib = residue_ids(varlen_lengths(calib_seqs, seed + 1), seed + 2)
    stats = m.calibrate(calib, 99.9)
    m.apply_smoothquant(stats, alpha, on_device=True)
    m.quantize_weights(on_device=True)
    return m


def quantized_650m(seed: int = 0, device: int = 0, calib_seqs: int = 32, alpha: float = 0.5,
                   num_layers: int | None = None) -> Model:
    """BASELINE config 3 weights (ESM-2 650M)."""
    return quantized_model("esm2_650m", seed, device, calib_seqs, alpha, num_layers)
