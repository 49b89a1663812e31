"""esm_b200.Model -- the reference's Python `esm_cpp.Model` API over the
device-resident B200 engine (python/esm_cpp/_core.cpp:79-525,
_core.pyi:49-80): load_from_safetensors / load_from_gguf / load,
quantize_weights, apply_smoothquant, forward_with_observer, forward,
forward_packed, forward_scheduled, save_to_gguf.

Weights stay on the host (numpy) until the first forward, which uploads one
replica to the model's device through the C ABI; every forward then runs on
the GPU.  There is no CPU execution path.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib
from .io import read_gguf, read_safetensors, write_gguf, write_safetensors
from .prep import migrate_smoothquant, quantize_weight

F32 = np.float32
VOCAB_SIZE = 33        # tokenizer.h:31
MASK_ID = 32           # tokenizer.h:30
CLS_ID, PAD_ID, EOS_ID = 0, 1, 2
LINEARS = ("q", "k", "v", "out", "fc1", "fc2")
SITES = ("attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu")


@dataclass
class Config:
    """model.h:22-48 Config."""
    num_hidden_layers: int
    hidden_size: int
    num_attention_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int = VOCAB_SIZE
    layer_norm_eps: float = 1e-5
    token_dropout: bool = True
    mask_token_id: int = MASK_ID
    weights_quantized: bool = False
    first_block_fc1_fp16: bool = False
    lm_head_dense_quantized: bool = False


def _hf_layer_keys(i: int) -> dict:
    p = f"esm.encoder.layer.{i}"
    return {
        "attn_ln_w": f"{p}.attention.LayerNorm.weight", "attn_ln_b": f"{p}.attention.LayerNorm.bias",
        "q_w": f"{p}.attention.self.query.weight", "q_b": f"{p}.attention.self.query.bias",
        "k_w": f"{p}.attention.self.key.weight", "k_b": f"{p}.attention.self.key.bias",
        "v_w": f"{p}.attention.self.value.weight", "v_b": f"{p}.attention.self.value.bias",
        "out_w": f"{p}.attention.output.dense.weight", "out_b": f"{p}.attention.output.dense.bias",
        "ffn_ln_w": f"{p}.LayerNorm.weight", "ffn_ln_b": f"{p}.LayerNorm.bias",
        "fc1_w": f"{p}.intermediate.dense.weight", "fc1_b": f"{p}.intermediate.dense.bias",
        "fc2_w": f"{p}.output.dense.weight", "fc2_b": f"{p}.output.dense.bias",
    }


_GGUF_LAYER = {
    "attn_ln_w": "attn_norm.weight", "attn_ln_b": "attn_norm.bias",
    "q_w": "attn_q.weight", "q_b": "attn_q.bias", "k_w": "attn_k.weight", "k_b": "attn_k.bias",
    "v_w": "attn_v.weight", "v_b": "attn_v.bias",
    "out_w": "attn_output.weight", "out_b": "attn_output.bias",
    "ffn_ln_w": "ffn_norm.weight", "ffn_ln_b": "ffn_norm.bias",
    "fc1_w": "ffn_up.weight", "fc1_b": "ffn_up.bias", "fc2_w": "ffn_down.weight", "fc2_b": "ffn_down.bias",
}
_GGUF_HEAD = {
    "final_ln_w": "enc_norm.weight", "final_ln_b": "enc_norm.bias",
    "lm_dense_w": "lm_head.weight", "lm_dense_b": "lm_head.bias",
    "lm_ln_w": "lm_head_norm.weight", "lm_ln_b": "lm_head_norm.bias", "lm_bias": "output.bias",
}
_HF_HEAD = {
    "final_ln_w": "esm.encoder.emb_layer_norm_after.weight",
    "final_ln_b": "esm.encoder.emb_layer_norm_after.bias",
    "lm_dense_w": "lm_head.dense.weight", "lm_dense_b": "lm_head.dense.bias",
    "lm_ln_w": "lm_head.layer_norm.weight", "lm_ln_b": "lm_head.layer_norm.bias",
    "lm_bias": "lm_head.bias",
}


class ActivationObserver:
    """observer.h ActivationObserver over the native esmcu_observer: per-site
    reservoirs of at most 65536 |values| (Algorithm R, std::mt19937 seeded
    0xc1b1ce), fed by Model.forward_with_observer / Model.calibrate in the
    order the reference's ForwardWithObserver calls would feed them."""

    def __init__(self):
        h = C.c_void_p()
        _lib.call("esmcu_observer_create", C.byref(h))
        self._h = h

    @property
    def handle(self):
        return self._h

    def observe(self, site_key: str, values) -> None:
        """ActivationObserver::Observe on host values."""
        v = np.ascontiguousarray(values, F32).ravel()
        _lib.call("esmcu_observer_observe", self._h, site_key.encode(), v.ctypes.data, v.size)

    def percentile(self, pctile: float) -> dict:
        """ActivationObserver::Percentile: {site key: pctile-th percentile}."""
        out = {}
        n = _lib.lib().esmcu_observer_num_sites(self._h)
        key, val = C.c_char_p(), C.c_float()
        for i in range(max(n, 0)):
            _lib.call("esmcu_observer_site", self._h, i, float(pctile), C.byref(key), C.byref(val),
                      None)
            out[key.value.decode()] = float(val.value)
        return out

    def clear(self) -> None:
        _lib.call("esmcu_observer_clear", self._h)

    def __del__(self):
        try:
            if self._h is not None:
                _lib.lib().esmcu_observer_destroy(self._h)
                self._h = None
        except Exception:
            pass


class Model:
    def __init__(self, config: Config, embed, layers, head, device: int = 0,
                 act_quant: str = "per_tensor"):
        self._cfg = config
        self.embed = np.ascontiguousarray(embed, F32)
        self.layers = layers
        self.head = head
        self.device = device
        self.act_quant = act_quant
        self._ctx = None
        self._dev = None
        self._dirty = True

    # ------------------------------------------------------------- loading
    @staticmethod
    def load_from_safetensors(path, device: int = 0) -> "Model":
        """model.cpp:65-147: config inferred from tensor shapes."""
        t = read_safetensors(path)
        embed = t["esm.embeddings.word_embeddings.weight"].astype(F32)
        V, d = embed.shape
        if V != VOCAB_SIZE:
            raise RuntimeError(f"vocab size mismatch: expected {VOCAB_SIZE} got {V}")
        dh = 2 * t["esm.encoder.layer.0.attention.self.rotary_embeddings.inv_freq"].shape[0]
        if d % dh:
            raise RuntimeError("hidden_size not divisible by head_dim")
        n = 0
        while f"esm.encoder.layer.{n}.attention.LayerNorm.weight" in t:
            n += 1
        if n == 0:
            raise RuntimeError("no encoder layers found")
        ffn = t["esm.encoder.layer.0.intermediate.dense.weight"].shape[0]
        cfg = Config(n, d, d // dh, dh, ffn)
        layers = [{k: t[v].astype(F32) for k, v in _hf_layer_keys(i).items()} for i in range(n)]
        head = {k: t[v].astype(F32) for k, v in _HF_HEAD.items()}
        return Model(cfg, embed, layers, head, device)

    @staticmethod
    def load_from_gguf(path, device: int = 0) -> "Model":
        """model.cpp:206-298 incl. Q8_ESM blobs (model.cpp:174-195)."""
        meta, t = read_gguf(path)
        if meta.get("general.architecture") != "esm":
            raise RuntimeError("gguf: not an esm-arch file (general.architecture must be 'esm')")
        cfg = Config(int(meta["esm.block_count"]), int(meta["esm.embedding_length"]),
                     int(meta["esm.attention.head_count"]), int(meta["esm.rope.dimension_count"]),
                     int(meta["esm.feed_forward_length"]),
                     layer_norm_eps=float(meta.get("esm.attention.layer_norm_epsilon", 1e-5)),
                     weights_quantized=bool(meta.get("esm.weights_quantized", False)),
                     first_block_fc1_fp16=bool(meta.get("esm.first_block_fc1_fp16", False)))
        layers = []
        for i in range(cfg.num_hidden_layers):
            lw = {}
            for k, g in _GGUF_LAYER.items():
                v = t[f"blk.{i}.{g}"]
                if isinstance(v, tuple):
                    lw[k + "q"], lw[k + "s"] = v
                else:
                    lw[k] = v
            layers.append(lw)
        head = {k: t[g] for k, g in _GGUF_HEAD.items()}
        return Model(cfg, t["token_embd.weight"], layers, head, device)

    @staticmethod
    def load(path, device: int = 0) -> "Model":
        """model.cpp:300-303: GGUF by magic, safetensors otherwise."""
        with open(path, "rb") as f:
            magic = f.read(4)
        if magic == b"GGUF":
            return Model.load_from_gguf(path, device)
        return Model.load_from_safetensors(path, device)

    def save_to_gguf(self, path) -> None:
        """model.cpp:562-725."""
        c = self._cfg
        meta = {
            "general.architecture": "esm", "general.alignment": 32,
            "general.file_type": 2 if c.weights_quantized else 1,
            "esm.block_count": c.num_hidden_layers, "esm.embedding_length": c.hidden_size,
            "esm.feed_forward_length": c.intermediate_size,
            "esm.attention.head_count": c.num_attention_heads,
            "esm.attention.head_count_kv": c.num_attention_heads,
            "esm.attention.layer_norm_epsilon": float(c.layer_norm_eps),
            "esm.rope.dimension_count": c.head_dim, "esm.context_length": 1024,
            "esm.gguf_writer": "esm_b200 0.1.0",
            "esm.weights_quantized": bool(c.weights_quantized),
            "esm.first_block_fc1_fp16": bool(c.first_block_fc1_fp16),
        }
        tensors = [("token_embd.weight", self.embed)]
        for i, lw in enumerate(self.layers):
            for k, g in _GGUF_LAYER.items():
                if k.endswith("_w") and k[:-2] in LINEARS and c.weights_quantized:
                    tensors.append((f"blk.{i}.{g}", (lw[k + "q"], lw[k + "s"])))
                else:
                    tensors.append((f"blk.{i}.{g}", lw[k]))
        for k, g in _GGUF_HEAD.items():
            tensors.append((g, self.head[k]))
        write_gguf(path, meta, tensors)

    def save_to_safetensors(self, path) -> None:
        """FP32 HF-keyed file (the layout load_from_safetensors reads)."""
        if self._cfg.weights_quantized:
            raise RuntimeError("safetensors holds FP32 weights; save a quantised model to GGUF")
        c = self._cfg
        out = {"esm.embeddings.word_embeddings.weight": self.embed}
        half = c.head_dim // 2
        inv = (1.0 / (10000.0 ** (np.arange(half, dtype=np.float64) * 2 / c.head_dim))).astype(F32)
        out["esm.encoder.layer.0.attention.self.rotary_embeddings.inv_freq"] = inv
        for i, lw in enumerate(self.layers):
            for k, key in _hf_layer_keys(i).items():
                out[key] = lw[k]
        for k, key in _HF_HEAD.items():
            out[key] = self.head[k]
        write_safetensors(path, out)

    # ----------------------------------------------------------- config
    @property
    def config(self) -> Config:
        return self._cfg

    @property
    def num_threads(self) -> int:
        return 1

    def set_act_quant(self, mode: str) -> None:
        if mode not in ("per_tensor", "per_token"):
            raise ValueError("act_quant must be 'per_tensor' or 'per_token'")
        self.act_quant = mode
        self._dirty = True

    def set_math_mode(self, mode: str) -> None:
        """"default" or "avx512": with "avx512" this model's forwards run
        LayerNorm, GELU and attention with the reference's default x86
        arithmetic bit for bit (esmcu_math_mode ESMCU_MATH_AVX512), so a W8A8
        forward reproduces the reference's default path layer by layer."""
        self._ensure_device()
        _lib.call("esmcu_set_math_mode", self._ctx, _lib.MATH_MODES[mode])

    def set_first_block_fc1_fp16(self, enabled: bool) -> None:
        """Config::first_block_fc1_fp16: round layer 0's fc1 input to fp16
        precision (model.cpp:1031-1033); saved as esm.first_block_fc1_fp16."""
        self._cfg.first_block_fc1_fp16 = bool(enabled)
        self._dirty = True

    # ------------------------------------------------------- quantisation
    def quantize_weights(self, on_device: bool = False) -> None:
        """model.cpp:1470-1494: per-layer Linears to per-channel int8, and
        lm_head.dense too when ESM_QUANTIZE_LM_HEAD is set to anything but
        "", "0" or "off" (model.cpp:1487-1492; the LM head's LayerNorm and the
        tied decoder stay FP32).  on_device=True quantises the FP32 replica
        already in HBM in place (esmcu_model_quantize_weights) and reads the
        codes back for the host copy; the codes and scales are the same bits
        as numpy's (and the reference's)."""
        if self._cfg.weights_quantized:
            return
        env = os.environ.get("ESM_QUANTIZE_LM_HEAD")
        lm_head = bool(env) and env not in ("0", "off")
        if on_device:
            self._ensure_device()
            _lib.call("esmcu_model_quantize_weights", self._dev, int(lm_head))
            self._pull_layers(quantized=True)
            if lm_head:
                d = self._cfg.hidden_size
                wq, ws = np.empty((d, d), np.int8), np.empty(d, F32)
                _lib.call("esmcu_model_get_head_int8", self._dev, wq.ctypes.data, ws.ctypes.data)
                self.head["lm_dense_wq"], self.head["lm_dense_ws"] = wq, ws
                self._cfg.lm_head_dense_quantized = True
            self._cfg.weights_quantized = True
            return  # the device replica is already the quantised model
        for lw in self.layers:
            for n in LINEARS:
                q, s = quantize_weight(lw[n + "_w"])
                lw[n + "_wq"], lw[n + "_ws"] = q, s
        if lm_head:
            self.head["lm_dense_wq"], self.head["lm_dense_ws"] = quantize_weight(self.head["lm_dense_w"])
            self._cfg.lm_head_dense_quantized = True
        self._cfg.weights_quantized = True
        self._dirty = True

    def apply_smoothquant(self, act_stats: dict, alpha: float, on_device: bool = False) -> None:
        """model.cpp:1462-1468 -> smoothquant.cpp:100-185 (FP32 weights).
        on_device=True migrates the FP32 replica in HBM
        (esmcu_model_apply_smoothquant) and reads the migrated weights back;
        the result is the same bits either way."""
        if self._cfg.weights_quantized:
            raise RuntimeError("apply_smoothquant runs on FP32 weights, before quantize_weights")
        if on_device:
            self._ensure_device()
            n = self._cfg.num_hidden_layers
            st = np.array([act_stats.get(f"layer{i}.{SITES[j]}", 0.0) for i in range(n) for j in range(4)],
                          F32)
            _lib.call("esmcu_model_apply_smoothquant", self._dev, st.ctypes.data, float(alpha))
            self._pull_layers(quantized=False)
            return
        for i, lw in enumerate(self.layers):
            migrate_smoothquant(lw, act_stats, i, alpha)
        self._dirty = True

    def _pull_layers(self, quantized: bool) -> None:
        """Copies the device replica's layers into the host arrays (LN,
        biases, and FP32 or int8 weights)."""
        c = self._cfg
        d, f = c.hidden_size, c.intermediate_size
        shapes = {"q": (d, d), "k": (d, d), "v": (d, d), "out": (d, d), "fc1": (f, d), "fc2": (d, f)}
        for i, lw in enumerate(self.layers):
            buf = _lib.LayerBuffers()
            keep = {}

            def arr(name, shape, dtype, ptr_t):
                a = np.empty(shape, dtype)
                keep[name] = a
                setattr(buf, name, C.cast(a.ctypes.data, ptr_t))

            for name in ("attn_ln_w", "attn_ln_b", "ffn_ln_w", "ffn_ln_b"):
                arr(name, (d,), F32, _lib._FP)
            for n, shp in shapes.items():
                arr(n + "_b", (shp[0],), F32, _lib._FP)
                if quantized:
                    arr(n + "_wq", shp, np.int8, _lib._I8P)
                    arr(n + "_ws", (shp[0],), F32, _lib._FP)
                else:
                    arr(n + "_w", shp, F32, _lib._FP)
            _lib.call("esmcu_model_get_layer", self._dev, i, C.byref(buf))
            lw.update(keep)

    def calibrate(self, sequences, pctile: float = 99.9) -> dict:
        """quantize.py calibrate (python/esm_cpp/quantize.py:35-47): every
        sequence observed through ForwardWithObserver, then Percentile.  The
        sequences run as one packed forward, which observes the same values
        in the same order as one call per sequence."""
        obs = ActivationObserver()
        seqs = [np.ascontiguousarray(s, np.int32) for s in sequences]
        if seqs:
            ids, cu = np.concatenate(seqs), np.concatenate(
                [[0], np.cumsum([len(s) for s in seqs])]).astype(np.int32)
            self._forward_observed(ids, cu, obs, None)
        return obs.percentile(pctile)

    def forward_with_observer(self, input_ids, attention_mask, observer: ActivationObserver):
        """Model::ForwardWithObserver (model.cpp:1084-1090): logits [L, V] of one
        sequence, its four Linear inputs per layer fed to `observer`."""
        if attention_mask is not None and not np.all(np.asarray(attention_mask) == 1):
            raise NotImplementedError("calibration takes unpadded sequences")
        ids = np.ascontiguousarray(input_ids, np.int32)
        logits = np.empty((ids.shape[0], self._cfg.vocab_size), F32)
        self._forward_observed(ids, np.array([0, ids.shape[0]], np.int32), observer, logits)
        return logits

    def _forward_observed(self, ids, cu, observer, logits):
        if self._cfg.weights_quantized:
            raise RuntimeError("calibrate before quantize_weights")
        self._ensure_device()
        _lib.call("esmcu_model_forward_observed", self._dev, observer.handle, ids.ctypes.data,
                  ids.shape[0], cu.ctypes.data, cu.shape[0] - 1,
                  None if logits is None else logits.ctypes.data)

    # ------------------------------------------------------------- device
    def _ensure_device(self):
        L = _lib.lib()
        if self._ctx is None:
            ctx = C.c_void_p()
            _lib.call("esmcu_open", self.device, C.byref(ctx))
            self._ctx = ctx
        if not self._dirty and self._dev is not None:
            return
        if self._dev is not None:
            L.esmcu_model_destroy(self._dev)
            self._dev = None
        c = self._cfg
        cfg = _lib.Config(c.num_hidden_layers, c.hidden_size, c.num_attention_heads, c.head_dim,
                          c.intermediate_size, c.vocab_size, float(c.layer_norm_eps),
                          c.mask_token_id, int(c.weights_quantized),
                          _lib.ACT_PER_TOKEN if self.act_quant == "per_token" else _lib.ACT_PER_TENSOR)
        dev = C.c_void_p()
        _lib.call("esmcu_model_create", self._ctx, C.byref(cfg), C.byref(dev))
        self._dev = dev
        keep = []

        def fp(a, dtype=F32):
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        _lib.call("esmcu_model_set_embeddings", dev, fp(self.embed))
        for i, lw in enumerate(self.layers):
            w = _lib.LayerWeights()
            for name in ("attn_ln_w", "attn_ln_b", "ffn_ln_w", "ffn_ln_b"):
                setattr(w, name, C.cast(fp(lw[name]), _lib._FP))
            for n in LINEARS:
                setattr(w, n + "_b", C.cast(fp(lw[n + "_b"]), _lib._FP))
                if c.weights_quantized:
                    setattr(w, n + "_wq", C.cast(fp(lw[n + "_wq"], np.int8), _lib._I8P))
                    setattr(w, n + "_ws", C.cast(fp(lw[n + "_ws"]), _lib._FP))
                else:
                    setattr(w, n + "_w", C.cast(fp(lw[n + "_w"]), _lib._FP))
            _lib.call("esmcu_model_set_layer", dev, i, C.byref(w))
        h = self.head
        _lib.call("esmcu_model_set_head", dev, fp(h["final_ln_w"]), fp(h["final_ln_b"]),
                  fp(h["lm_dense_w"]), fp(h["lm_dense_b"]), fp(h["lm_ln_w"]), fp(h["lm_ln_b"]),
                  fp(h["lm_bias"]))
        if c.first_block_fc1_fp16:
            _lib.call("esmcu_model_set_first_block_fc1_fp16", dev, 1)
        if c.lm_head_dense_quantized:
            _lib.call("esmcu_model_set_head_int8", dev, fp(h["lm_dense_wq"], np.int8),
                      fp(h["lm_dense_ws"]))
        self._dirty = False

    def close(self) -> None:
        if self._dev is not None:
            _lib.lib().esmcu_model_destroy(self._dev)
            self._dev = None
        if self._ctx is not None:
            _lib.lib().esmcu_close(self._ctx)
            self._ctx = None
        self._dirty = True

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        self._ensure_device()
        return self._dev

    def last_launch_count(self) -> int:
        return _lib.lib().esmcu_model_last_launch_count(self._dev) if self._dev else 0

    def set_profiling(self, on: bool) -> None:
        self._ensure_device()
        _lib.call("esmcu_model_set_profiling", self._dev, int(on))

    def profile(self) -> dict:
        names = (C.c_char_p * 64)()
        ms = np.zeros(64, F32)
        n = _lib.lib().esmcu_model_profile(self._dev, names, ms.ctypes.data, 64)
        return {names[i].decode(): float(ms[i]) for i in range(max(n, 0))}

    # ------------------------------------------------------------ forward
    def forward_packed(self, packed_ids, cu_seqlens, packed_masks=None, out=None):
        """Model::ForwardPacked: list of [L_b, V] logits (or, with out=, the
        packed [T, V] array written in place)."""
        self._ensure_device()
        ids = np.ascontiguousarray(packed_ids, np.int32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        if ids.ndim != 1:
            raise ValueError("packed_ids must be a 1-D int32 array")
        if cu.ndim != 1 or cu.shape[0] < 2:
            raise ValueError("cu_seqlens must be a 1-D int32 array of size batch + 1")
        masks = None if packed_masks is None else np.ascontiguousarray(packed_masks, np.int32)
        if masks is not None and masks.shape != ids.shape:
            raise ValueError("packed_masks must be a 1-D int32 array of the same length as packed_ids")
        T, B, V = ids.shape[0], cu.shape[0] - 1, self._cfg.vocab_size
        logits = out if out is not None else np.empty((T, V), F32)
        _lib.call("esmcu_model_forward_packed", self._dev, ids.ctypes.data,
                  None if masks is None else masks.ctypes.data, T, cu.ctypes.data, B,
                  logits.ctypes.data)
        if out is not None:
            return out
        return [logits[cu[b]:cu[b + 1]] for b in range(B)]

    def forward_packed_device(self, d_ids, cu_seqlens, d_logits, d_masks=None):
        """Model::ForwardPacked on device tensors (esmcu_model_forward_packed_device):
        d_ids int32 [T] and d_logits float32 [T, V] (contiguous, on this model's
        GPU), cu_seqlens host int32 [B + 1].  Runs on torch's current stream
        of the device, so torch copies before and after it are ordered with
        it; nothing is synchronised."""
        import torch

        self._ensure_device()
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        T, V = int(cu[-1]), self._cfg.vocab_size
        if d_ids.dtype != torch.int32 or d_ids.numel() != T or not d_ids.is_contiguous():
            raise ValueError("d_ids must be a contiguous int32 tensor of cu_seqlens[-1] elements")
        if d_logits.dtype != torch.float32 or tuple(d_logits.shape) != (T, V) or not d_logits.is_contiguous():
            raise ValueError("d_logits must be a contiguous float32 tensor [T, vocab]")
        _lib.call("esmcu_set_stream", self._ctx, _lib.torch_stream_handle(self.device))
        _lib.call("esmcu_model_forward_packed_device", self._dev, C.c_void_p(d_ids.data_ptr()),
                  None if d_masks is None else C.c_void_p(d_masks.data_ptr()), T, cu.ctypes.data,
                  cu.shape[0] - 1, C.c_void_p(d_logits.data_ptr()))
        return d_logits

    def forward(self, input_ids, attention_mask=None):
        ids = np.ascontiguousarray(input_ids, np.int32)
        if ids.ndim != 1:
            raise ValueError("input_ids must be a 1-D int32 array")
        if ids.shape[0] == 0:
            return np.empty((0, self._cfg.vocab_size), F32)
        return self.forward_packed(ids, np.array([0, ids.shape[0]], np.int32), attention_mask)[0]

    def forward_packed_hidden_states(self, packed_ids, cu_seqlens, packed_masks=None):
        """ForwardPackedInto with hidden_packed_out (model.cpp:1142-1189) on a
        packed batch: (logits [T, V], hidden [num_layers + 1, T, d]) with
        hidden[0] the embedding output, hidden[i] layer i-1's output and
        hidden[num_layers] the final LayerNorm's output."""
        self._ensure_device()
        ids = np.ascontiguousarray(packed_ids, np.int32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        if ids.ndim != 1:
            raise ValueError("packed_ids must be a 1-D int32 array")
        if cu.ndim != 1 or cu.shape[0] < 2:
            raise ValueError("cu_seqlens must be a 1-D int32 array of size batch + 1")
        masks = None if packed_masks is None else np.ascontiguousarray(packed_masks, np.int32)
        if masks is not None and masks.shape != ids.shape:
            raise ValueError("packed_masks must be a 1-D int32 array of the same length as packed_ids")
        c = self._cfg
        T, B = ids.shape[0], cu.shape[0] - 1
        logits = np.empty((T, c.vocab_size), F32)
        hidden = np.empty((c.num_hidden_layers + 1, T, c.hidden_size), F32)
        if T == 0:
            return logits, hidden
        _lib.call("esmcu_model_forward_hidden_states", self._dev, ids.ctypes.data,
                  None if masks is None else masks.ctypes.data, T, cu.ctypes.data, B,
                  logits.ctypes.data, hidden.ctypes.data)
        return logits, hidden

    def forward_with_hidden_states(self, input_ids, attention_mask=None):
        """Model::ForwardWithHiddenStates (model.h:185-191; the Python binding
        forward_with_hidden_states, _core.cpp:511-524): (logits [L, V],
        [hidden_state_0, ..., hidden_state_N]), N = num_hidden_layers,
        hidden_state_0 post-embed, hidden_state_N post-final-LN, each [L, d]."""
        ids = np.ascontiguousarray(input_ids, np.int32)
        if ids.ndim != 1:
            raise ValueError("input_ids must be a 1-D int32 array")
        logits, hidden = self.forward_packed_hidden_states(
            ids, np.array([0, ids.shape[0]], np.int32), attention_mask)
        return logits, [hidden[i] for i in range(hidden.shape[0])]

    @staticmethod
    def _concat_sequences(input_ids, attention_masks):
        """(lens [n], ids_concat, masks_concat or None) of a list of sequences."""
        seqs = [np.ascontiguousarray(a, np.int32) for a in input_ids]
        for a in seqs:
            if a.ndim != 1:
                raise ValueError("each input_ids entry must be a 1-D int32 array")
        n = len(seqs)
        lens = np.array([a.shape[0] for a in seqs], np.int32)
        ids = np.concatenate(seqs) if n and lens.sum() else np.zeros(0, np.int32)
        masks = None
        if attention_masks is not None:
            if len(attention_masks) != n:
                raise ValueError("attention_masks length must match input_ids length")
            ms = [np.ascontiguousarray(m, np.int32) for m in attention_masks]
            for m, a in zip(ms, seqs):
                if m.shape != a.shape:
                    raise ValueError("attention_mask[i] must be a 1-D int32 array of the same length as input_ids[i]")
            masks = np.concatenate(ms)
        return lens, ids, masks

    def forward_scheduled(self, input_ids, attention_masks=None, imbalance_threshold: float = 1.2,
                          max_batch_size: int = 256):
        """Model::ForwardScheduled: logits in input order."""
        self._ensure_device()
        lens, ids, masks = self._concat_sequences(input_ids, attention_masks)
        n = lens.shape[0]
        if n == 0:
            return []
        V = self._cfg.vocab_size
        logits = np.empty((int(lens.sum()), V), F32)
        _lib.call("esmcu_model_forward_scheduled", self._dev, ids.ctypes.data, lens.ctypes.data,
                  None if masks is None else masks.ctypes.data, n, float(imbalance_threshold),
                  int(max_batch_size), logits.ctypes.data)
        off = np.concatenate([[0], np.cumsum(lens)])
        return [logits[off[i]:off[i + 1]] for i in range(n)]

    def masked_marginals(self, input_ids, rows, attention_masks=None,
                         imbalance_threshold: float = 1.2, max_batch_size: int = 256):
        """log_softmax(forward_scheduled(input_ids)[i][rows[i]]) for every i, as
        one [n, V] array, without the full logits: the LM head runs on the n
        scored rows only and the log-softmax on the device
        (esmcu_model_masked_marginals; eval/proteingym.py:84-98 takes these
        rows of the masked copies' logits)."""
        self._ensure_device()
        lens, ids, masks = self._concat_sequences(input_ids, attention_masks)
        n = lens.shape[0]
        r = np.ascontiguousarray(rows, np.int32)
        if r.shape != (n,):
            raise ValueError("rows must hold one row index per sequence")
        V = self._cfg.vocab_size
        out = np.empty((n, V), F32)
        if n == 0:
            return out
        _lib.call("esmcu_model_masked_marginals", self._dev, ids.ctypes.data, lens.ctypes.data,
                  None if masks is None else masks.ctypes.data, r.ctypes.data, n,
                  float(imbalance_threshold), int(max_batch_size), out.ctypes.data)
        return out


def forward_scheduled_multi(models, input_ids, imbalance_threshold: float = 1.2,
                            max_batch_size: int = 256):
    """ForwardScheduled across several per-device replicas in one process
    (one host thread per device; groups assigned longest-processing-time)."""
    for m in models:
        m._ensure_device()
    seqs = [np.ascontiguousarray(a, np.int32) for a in input_ids]
    lens = np.array([a.shape[0] for a in seqs], np.int32)
    ids = np.concatenate(seqs)
    V = models[0].config.vocab_size
    logits = np.empty((int(lens.sum()), V), F32)
    handles = (C.c_void_p * len(models))(*[m._dev.value for m in models])
    _lib.call("esmcu_forward_scheduled_multi", handles, len(models), ids.ctypes.data,
              lens.ctypes.data, None, len(seqs), float(imbalance_threshold), int(max_batch_size),
              logits.ctypes.data)
    off = np.concatenate([[0], np.cumsum(lens)])
    return [logits[off[i]:off[i + 1]] for i in range(len(seqs))]
