"""Offline weight preparation (host, numpy): the reference's load-time
quantisation and SmoothQuant migration, restated for this package.

  quantize_weight      pack.cpp:149-177   per-output-channel symmetric int8,
                                           scale = rowmax/127, an all-zero
                                           row keeps scale 0.
  smoothquant_scales   smoothquant.cpp:49-74   s = P_X^a / P_W^(1-a),
                                           clamped to [1e-3, 1e3].
  migrate_smoothquant  smoothquant.cpp:100-185 three sites per layer; P_X is
                                           one per-tensor scalar broadcast to
                                           all channels (smoothquant.cpp:78-96).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def quantize_weight(w: np.ndarray):
    """[N, K] float32 -> (int8 [N, K], float32 scales [N]); bit-identical to
    quant::Quantize (IEEE float divides/multiplies, round-half-even)."""
    w = np.ascontiguousarray(w, F32)
    row_max = np.max(np.abs(w), axis=1).astype(F32) if w.shape[1] else np.zeros(w.shape[0], F32)
    scale = (row_max / F32(127.0)).astype(F32)
    q = np.zeros(w.shape, np.int8)
    nz = row_max != 0
    if nz.any():
        inv = (F32(1.0) / scale[nz]).astype(F32)
        v = np.rint((w[nz] * inv[:, None]).astype(F32))
        q[nz] = np.clip(v, -127, 127).astype(np.int8)
    scale[~nz] = 0.0
    return q, scale


_powf = None


def _c_powf():
    """The C library's powf, the function the reference's std::pow(float,
    float) calls (numpy's power rounds differently in the last ulp)."""
    global _powf
    if _powf is None:
        import ctypes
        import ctypes.util

        libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
        libm.powf.restype = ctypes.c_float
        libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
        _powf = libm.powf
    return _powf


def smoothquant_scales(p_x: np.ndarray, p_w: np.ndarray, alpha: float) -> np.ndarray:
    """smoothquant.cpp:49-74 channel by channel: s = powf(P_X, a) / powf(P_W,
    1 - a) in float, 1 where either input is not positive or s is not a
    positive finite number, clamped to [1e-3, 1e3]."""
    p_x = np.asarray(p_x, F32).ravel()
    p_w = np.asarray(p_w, F32).ravel()
    powf = _c_powf()
    a = float(F32(alpha))
    b = float(F32(1.0) - F32(alpha))
    s = np.ones(p_x.shape, F32)
    for k in range(p_x.size):
        px, pw = float(p_x[k]), float(p_w[k])
        if not (px > 0.0 and pw > 0.0):
            continue
        with np.errstate(all="ignore"):
            val = F32(powf(px, a)) / F32(powf(pw, b))
        if not np.isfinite(val) or val <= 0:
            continue
        s[k] = min(max(val, F32(1e-3)), F32(1e3))
    return s


def migrate_smoothquant(layer: dict, stats: dict, i: int, alpha: float) -> None:
    """In place on one layer dict (fp32 weights).  stats keys follow the
    reference's observer sites: layer<i>.attn_ln_output / attn_out /
    ffn_ln_output / inter_gelu."""
    pre = f"layer{i}"
    K = layer["attn_ln_w"].shape[0]
    # Site 1: attn_ln_output -> {Q, K, V}
    p_w = np.maximum.reduce([np.max(np.abs(layer[n]), axis=0) for n in ("q_w", "k_w", "v_w")])
    s = smoothquant_scales(np.full(K, stats.get(pre + ".attn_ln_output", 0.0), F32), p_w, alpha)
    layer["attn_ln_w"] = (layer["attn_ln_w"] / s).astype(F32)
    layer["attn_ln_b"] = (layer["attn_ln_b"] / s).astype(F32)
    for n in ("q_w", "k_w", "v_w"):
        layer[n] = (layer[n] * s[None, :]).astype(F32)
    # Site 2: attn_out -> out_proj (V output rows scaled down)
    Nv = layer["v_b"].shape[0]
    p_w = np.max(np.abs(layer["out_w"]), axis=0)
    s = smoothquant_scales(np.full(Nv, stats.get(pre + ".attn_out", 0.0), F32), p_w, alpha)
    layer["v_b"] = (layer["v_b"] / s).astype(F32)
    layer["v_w"] = (layer["v_w"] / s[:, None]).astype(F32)
    layer["out_w"] = (layer["out_w"] * s[None, :]).astype(F32)
    # Site 3: ffn_ln_output -> fc1
    Kf = layer["ffn_ln_w"].shape[0]
    p_w = np.max(np.abs(layer["fc1_w"]), axis=0)
    s = smoothquant_scales(np.full(Kf, stats.get(pre + ".ffn_ln_output", 0.0), F32), p_w, alpha)
    layer["ffn_ln_w"] = (layer["ffn_ln_w"] / s).astype(F32)
    layer["ffn_ln_b"] = (layer["ffn_ln_b"] / s).astype(F32)
    layer["fc1_w"] = (layer["fc1_w"] * s[None, :]).astype(F32)
    # inter_gelu -> fc2 is not migrated (GELU breaks the diagonal rescale).
