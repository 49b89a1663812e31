"""TEST INFRASTRUCTURE ONLY -- the checker, never the thing measured or shipped.

numpy bindings for
  * the C restatement of the reference's hot path (oracle/esm_oracle.c,
    built into oracle/_build/liboracle.so), and
  * the reference itself compiled from its own sources
    (oracle/_ref/libesmref.so, via oracle/ref_shim.cpp),
plus `forward_packed`, the reference's ForwardPackedInto (model.cpp:1093-1255)
composed from the restated ops.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm import this module.

Parity status: pinned (tests/test_oracle_pins.py checks the restatement
against oracle/_ref and the reference's unit-test known answers).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libesmref.so"
F32 = np.float32

_orc = None
_ref = None


def reference_source() -> Path | None:
    """The esm-cpp source tree: $REF_SRC when set (it must then hold
    src/model.cpp), else a checkout named `reference` beside this
    repository, else None (the prebuilt oracle/_ref, if any, is used)."""
    src = os.environ.get("REF_SRC")
    if src:
        if not Path(src, "src", "model.cpp").exists():
            raise FileNotFoundError(f"REF_SRC={src} has no src/model.cpp")
        return Path(src)
    sibling = HERE.parent.parent / "reference"
    return sibling if (sibling / "src" / "model.cpp").exists() else None


def build(ref: bool | None = None) -> None:
    """Builds liboracle.so (always) and libesmref.so (when the reference
    sources are found, see reference_source)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    src = reference_source()
    if ref is None:
        ref = src is not None
    if ref:
        if src is None:
            raise FileNotFoundError("the reference sources were not found: set REF_SRC")
        subprocess.run(["make", "-s", "-j8", "-C", str(HERE), "ref", f"REF_SRC={src}"], check=True)


_VP, _I, _F, _SZ = C.c_void_p, C.c_int, C.c_float, C.c_size_t
_ORC_SIGS = {
    "orc_quantize_weights": (None, [_VP, _I, _I, _VP, _VP]),
    "orc_absmax": (_F, [_VP, _SZ]),
    "orc_act_scale": (_F, [_F]),
    "orc_quantize_act": (None, [_VP, _SZ, _F, _VP]),
    "orc_quantize_act_per_token": (None, [_VP, _I, _I, _VP, _VP]),
    "orc_gemm_i8_s32": (None, [_VP, _VP, _VP, _I, _I, _I]),
    "orc_dequant": (None, [_VP, _VP, _F, _VP, _VP, _VP, _I, _I]),
    "orc_linear_f32": (None, [_VP, _VP, _VP, _VP, _I, _I, _I]),
    "orc_layernorm": (None, [_VP, _VP, _VP, _F, _VP, _I, _I]),
    "orc_gelu": (None, [_VP, _VP, _SZ]),
    "orc_residual_add": (None, [_VP, _VP, _SZ]),
    "orc_scale": (None, [_VP, _SZ, _F]),
    "orc_rope_build_tables": (None, [_I, _I, _VP, _VP]),
    "orc_rope_apply_varlen": (None, [_VP, _VP, _VP, _VP, _I, _I, _I, _I]),
    "orc_attention_varlen": (None, [_VP, _VP, _VP, _VP, _I, _I, _I, _VP]),
    "orc_embed": (None, [_VP, _I, _VP, _VP, _VP, _I, _I, _VP]),
    "orc_plan_batches": (_I, [_VP, _I, _F, _I, _VP, _VP]),
    "orc_layernorm_avx": (None, [_VP, _VP, _VP, _F, _VP, _I, _I]),
    "orc_gelu_avx": (None, [_VP, _VP, _SZ]),
    "orc_expf_libc": (_F, [_F]),
    "orc_attention_avx": (None, [_VP, _VP, _VP, _VP, _I, _I, _I, _VP, _VP]),
}
_REF_SIGS = {
    "ref_last_error": (C.c_char_p, []),
    "ref_host_isa": (C.c_char_p, []),
    "ref_current_isa": (C.c_char_p, []),
    "ref_force_isa": (None, [C.c_char_p]),
    "ref_num_threads": (_I, []),
    "ref_linear_f32": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_linear_f32_ref": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_linear_int8": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_linear_int8_vnni": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_linear_int8_amx": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_linear_int8_ref": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_quantize_weights": (_I, [_VP, _I, _I, _VP, _VP]),
    "ref_quantize_act": (_I, [_VP, _SZ, _F, _VP]),
    "ref_quantize_act_sym": (_I, [_VP, _SZ, _F, _VP]),
    "ref_quant_act_prefix": (_I, [_VP, _SZ, _VP, _VP]),
    "ref_layernorm": (_I, [_VP, _VP, _VP, _F, _VP, _I, _I]),
    "ref_layernorm_ref": (_I, [_VP, _VP, _VP, _F, _VP, _I, _I]),
    "ref_gelu": (_I, [_VP, _VP, _SZ]),
    "ref_gelu_ref": (_I, [_VP, _VP, _SZ]),
    "ref_residual_add": (_I, [_VP, _VP, _SZ]),
    "ref_scale": (_I, [_VP, _SZ, _F]),
    "ref_rope_build_tables": (_I, [_I, _I, _VP, _VP]),
    "ref_rope_apply_varlen": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_rope_apply_varlen_ref": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I]),
    "ref_attention_varlen": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _VP]),
    "ref_attention_varlen_ref": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _VP]),
    "ref_plan_batches": (_I, [_VP, _I, _F, _I, _VP, _VP]),
    "ref_batch_view_check": (_I, [_VP, _I, _VP, _I, _VP, _I, _I]),
    "ref_model_load": (_VP, [C.c_char_p]),
    "ref_model_free": (None, [_VP]),
    "ref_model_config": (_I, [_VP, _VP]),
    "ref_model_forward_packed": (_I, [_VP, _VP, _VP, _I, _VP, _I, _VP]),
    "ref_model_forward_scheduled": (_I, [_VP, _VP, _VP, _I, _F, _I, _VP]),
    "ref_model_forward_hidden": (_I, [_VP, _VP, _I, _VP, _VP]),
    "ref_model_calibrate_smoothquant": (_I, [_VP, _VP, _VP, _I, _F, _F]),
    "ref_model_quantize": (_I, [_VP]),
    "ref_model_save_gguf": (_I, [_VP, C.c_char_p]),
    "ref_observer_new": (_VP, []),
    "ref_observer_free": (None, [_VP]),
    "ref_observer_observe": (_I, [_VP, C.c_char_p, _VP, _SZ]),
    "ref_observer_percentile": (_I, [_VP, C.c_char_p, _F, _VP]),
    "ref_model_observe": (_I, [_VP, _VP, _VP, _I, _F, _VP]),
    "ref_model_apply_smoothquant": (_I, [_VP, _VP, _F]),
}


def _bind(L, sigs):
    for name, (res, args) in sigs.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


def orc():
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        _orc = _bind(C.CDLL(str(ORACLE_SO)), _ORC_SIGS)
    return _orc


def ref_available() -> bool:
    return REF_SO.exists()


def ref():
    """The reference compiled from its own sources (raises if not built)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (make -C oracle ref)")
        _ref = _bind(C.CDLL(str(REF_SO)), _REF_SIGS)
    return _ref


def ref_check(rc: int, what: str = "ref") -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: {ref().ref_last_error().decode()}")


def _a(x, dt=F32):
    return np.ascontiguousarray(x, dt)


# --------------------------------------------------------- restated ops
def quantize_weights(W):
    W = _a(W)
    N, K = W.shape
    q = np.zeros((N, K), np.int8)
    s = np.zeros(N, F32)
    orc().orc_quantize_weights(W.ctypes.data, N, K, q.ctypes.data, s.ctypes.data)
    return q, s


def act_scale_per_tensor(A) -> float:
    A = _a(A)
    return float(orc().orc_act_scale(orc().orc_absmax(A.ctypes.data, A.size)))


def quantize_act(A, scale: float):
    A = _a(A)
    q = np.zeros(A.shape, np.int8)
    orc().orc_quantize_act(A.ctypes.data, A.size, C.c_float(scale), q.ctypes.data)
    return q


def quantize_act_per_tensor(A):
    s = act_scale_per_tensor(A)
    return quantize_act(A, s), np.array([s], F32)


def quantize_act_per_token(A):
    A = _a(A)
    M, K = A.shape
    q = np.zeros((M, K), np.int8)
    s = np.zeros(M, F32)
    orc().orc_quantize_act_per_token(A.ctypes.data, M, K, q.ctypes.data, s.ctypes.data)
    return q, s


def gemm_i8_s32(q, W):
    q, W = _a(q, np.int8), _a(W, np.int8)
    M, K = q.shape
    N = W.shape[0]
    acc = np.zeros((M, N), np.int32)
    orc().orc_gemm_i8_s32(q.ctypes.data, W.ctypes.data, acc.ctypes.data, M, N, K)
    return acc


def dequant(acc, ws, a_scale, bias=None):
    acc, ws = _a(acc, np.int32), _a(ws)
    M, N = acc.shape
    a_scale = _a(np.atleast_1d(a_scale))
    row = a_scale if a_scale.size == M and M > 1 else None
    C_ = np.zeros((M, N), F32)
    b = None if bias is None else _a(bias)
    orc().orc_dequant(acc.ctypes.data, ws.ctypes.data, C.c_float(float(a_scale[0])),
                      None if row is None else row.ctypes.data,
                      None if b is None else b.ctypes.data, C_.ctypes.data, M, N)
    return C_


def linear_int8(A, Wq, ws, bias=None, per_token: bool = False):
    """W8A8 LinearInt8 (VNNI semantics: one scale over all M rows)."""
    q, s = quantize_act_per_token(A) if per_token else quantize_act_per_tensor(A)
    return dequant(gemm_i8_s32(q, Wq), ws, s, bias)


def linear_f32(A, W, bias=None):
    A, W = _a(A), _a(W)
    M, K = A.shape
    N = W.shape[0]
    out = np.zeros((M, N), F32)
    b = None if bias is None else _a(bias)
    orc().orc_linear_f32(A.ctypes.data, W.ctypes.data, None if b is None else b.ctypes.data,
                         out.ctypes.data, M, N, K)
    return out


def layernorm(x, g, b, eps=1e-5):
    x = _a(x)
    rows, d = x.shape
    out = np.zeros_like(x)
    orc().orc_layernorm(x.ctypes.data, _a(g).ctypes.data, _a(b).ctypes.data, C.c_float(eps),
                        out.ctypes.data, rows, d)
    return out


def gelu(x):
    x = _a(x)
    out = np.zeros_like(x)
    orc().orc_gelu(x.ctypes.data, out.ctypes.data, x.size)
    return out


def layernorm_avx(x, g, b, eps=1e-5):
    """LayerNormAvx512 (layernorm.cpp:59-149) bit for bit, d % 16 == 0."""
    x = _a(x)
    out = np.zeros_like(x)
    rows, d = x.shape
    orc().orc_layernorm_avx(x.ctypes.data, _a(g).ctypes.data, _a(b).ctypes.data, C.c_float(eps),
                            out.ctypes.data, rows, d)
    return out


def gelu_avx(x):
    """GeluAvx512 (gelu.cpp:48-148) bit for bit."""
    x = _a(x)
    out = np.zeros_like(x)
    orc().orc_gelu_avx(x.ctypes.data, out.ctypes.data, x.size)
    return out


def expf_libc(x) -> np.ndarray:
    """The C library's expf, restated (orc_expf_libc), elementwise."""
    x = _a(x).ravel()
    f = orc().orc_expf_libc
    return np.array([f(float(v)) for v in x], F32)


def attention_avx(q, k, v, cu, H, dh):
    """AttentionVarlenAvx512 (attention.cpp:230-437, 770-811) bit for bit."""
    q, k, v = _a(q), _a(k), _a(v)
    cu = _a(cu, np.int32)
    out = np.zeros_like(q)
    maxL = int(np.max(np.diff(cu))) if cu.size > 1 else 1
    scratch = np.zeros(max(maxL, 1) + 16, F32)
    orc().orc_attention_avx(q.ctypes.data, k.ctypes.data, v.ctypes.data, cu.ctypes.data,
                            cu.size - 1, H, dh, out.ctypes.data, scratch.ctypes.data)
    return out


def rope_build_tables(L, dh):
    c = np.zeros((L, dh), F32)
    s = np.zeros((L, dh), F32)
    orc().orc_rope_build_tables(L, dh, c.ctypes.data, s.ctypes.data)
    return c, s


def rope_apply_varlen(x, cos_t, sin_t, cu, H, dh, fused=True):
    x = _a(x).copy()
    cu = _a(cu, np.int32)
    orc().orc_rope_apply_varlen(x.ctypes.data, _a(cos_t).ctypes.data, _a(sin_t).ctypes.data,
                                cu.ctypes.data, cu.size - 1, H, dh, int(fused))
    return x


def round_bf16(x):
    """float32 -> nearest bfloat16 value (ties to even), kept as float32: the
    conversion of the reference's BF16 attention (attention.cpp:707-768,
    _mm512_cvtne2ps_pbh).  NaN stays NaN."""
    x = _a(x)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(F32)
    return np.where(np.isnan(x), x, r).astype(F32)


def attention_bf16_enabled(dh: int) -> bool:
    """ESM_AMX_ATTENTION (attention.cpp:686-700), for head dims % 32 == 0."""
    return dh % 32 == 0 and os.environ.get("ESM_AMX_ATTENTION", "") in ("on", "1", "true")


def attention_varlen(q, k, v, cu, H, dh, bf16: bool = False):
    """AttentionVarlenRef; with bf16, Q and K rounded to bfloat16 first (the
    reference's opt-in BF16 attention: exact bf16 products, fp32 sums)."""
    if bf16:
        q, k = round_bf16(q), round_bf16(k)
    q, k, v, cu = _a(q), _a(k), _a(v), _a(cu, np.int32)
    out = np.zeros_like(q)
    orc().orc_attention_varlen(q.ctypes.data, k.ctypes.data, v.ctypes.data, cu.ctypes.data,
                               cu.size - 1, H, dh, out.ctypes.data)
    return out


def embed(E, ids, cu, masks=None, mask_id=32):
    E, ids, cu = _a(E), _a(ids, np.int32), _a(cu, np.int32)
    d = E.shape[1]
    out = np.zeros((ids.size, d), F32)
    m = None if masks is None else _a(masks, np.int32)
    orc().orc_embed(E.ctypes.data, d, ids.ctypes.data, None if m is None else m.ctypes.data,
                    cu.ctypes.data, cu.size - 1, mask_id, out.ctypes.data)
    return out


def plan_batches(lengths, threshold=1.2, max_batch=256):
    lens = _a(lengths, np.int32)
    n = lens.size
    order = np.zeros(max(n, 1), np.int32)
    sizes = np.zeros(max(n, 1), np.int32)
    g = orc().orc_plan_batches(lens.ctypes.data, n, C.c_float(threshold), max_batch,
                               order.ctypes.data, sizes.ctypes.data)
    out, p = [], 0
    for i in range(g):
        out.append(order[p:p + sizes[i]].tolist())
        p += sizes[i]
    return out


def forward_packed(model, ids, cu, masks=None, per_token: bool = False, hidden=None):
    """ForwardPackedInto (model.cpp:1093-1255) + TransformerBlock
    (model.cpp:932-1066) composed from the restated ops; `model` is an
    esm_b200.Model (host numpy weights).  Returns packed logits [T, V].
    With a list as `hidden`, it receives hidden_packed_out (model.cpp:
    1142-1189): the embedding output, each layer's output, and the final
    LayerNorm's output in place of the last layer's (num_layers + 1 [T, d])."""
    c = model.config
    d, H, dh = c.hidden_size, c.num_attention_heads, c.head_dim
    ids, cu = _a(ids, np.int32), _a(cu, np.int32)
    T = ids.size
    maxL = int(np.max(np.diff(cu))) if cu.size > 1 else 0
    h = embed(model.embed, ids, cu, masks, c.mask_token_id)
    if hidden is not None:
        hidden.clear()
        hidden.append(h.copy())
    cos_t, sin_t = rope_build_tables(max(maxL, 1), dh)
    qs = F32(1.0) / F32(np.sqrt(F32(dh)))

    def lin(x, lw, n):
        if c.weights_quantized:
            return linear_int8(x, lw[n + "_wq"], lw[n + "_ws"], lw[n + "_b"], per_token)
        return linear_f32(x, lw[n + "_w"], lw[n + "_b"])

    for li, lw in enumerate(model.layers):
        ln = layernorm(h, lw["attn_ln_w"], lw["attn_ln_b"], c.layer_norm_eps)
        q = lin(ln, lw, "q")
        k = lin(ln, lw, "k")
        v = lin(ln, lw, "v")
        q = (q * qs).astype(F32)
        q = rope_apply_varlen(q, cos_t, sin_t, cu, H, dh, fused=True)
        k = rope_apply_varlen(k, cos_t, sin_t, cu, H, dh, fused=True)
        att = attention_varlen(q, k, v, cu, H, dh, bf16=attention_bf16_enabled(dh))
        h = (h + lin(att, lw, "out")).astype(F32)
        ln = layernorm(h, lw["ffn_ln_w"], lw["ffn_ln_b"], c.layer_norm_eps)
        if li == 0 and getattr(c, "first_block_fc1_fp16", False):
            ln = ln.astype(np.float16).astype(F32)  # model.cpp:1031-1033, RNE
        inter = gelu(lin(ln, lw, "fc1"))
        h = (h + lin(inter, lw, "fc2")).astype(F32)
        if hidden is not None:
            hidden.append(h.copy())
    hd = model.head
    fl = layernorm(h, hd["final_ln_w"], hd["final_ln_b"], c.layer_norm_eps)
    if hidden is not None:
        hidden[-1] = fl.copy()
    if getattr(c, "lm_head_dense_quantized", False):  # LinearInt8 (model.cpp:1209-1211)
        g = gelu(linear_int8(fl, hd["lm_dense_wq"], hd["lm_dense_ws"], hd["lm_dense_b"], per_token))
    else:
        g = gelu(linear_f32(fl, hd["lm_dense_w"], hd["lm_dense_b"]))
    lm = layernorm(g, hd["lm_ln_w"], hd["lm_ln_b"], c.layer_norm_eps)
    return linear_f32(lm, model.embed, hd["lm_bias"])


def forward_scheduled(model, seqs, threshold=1.2, max_batch=256, per_token: bool = False):
    """Model::ForwardScheduled (model.cpp:1298-1421): PlanBatches groups,
    each packed and run through forward_packed; logits per sequence in
    caller order.  (The W8A8 per-tensor activation scale is an absmax over
    a group's rows, so the grouping is part of the result.)"""
    out = [None] * len(seqs)
    for g in plan_batches([len(s) for s in seqs], threshold, max_batch):
        ids = np.concatenate([_a(seqs[i], np.int32) for i in g])
        cu = np.concatenate([[0], np.cumsum([len(seqs[i]) for i in g])]).astype(np.int32)
        lg = forward_packed(model, ids, cu, per_token=per_token)
        for j, i in enumerate(g):
            out[i] = lg[cu[j]:cu[j + 1]]
    return out


def log_softmax_at(row, token: int) -> float:
    """eval/proteingym.py:48-50, numpy float32 as there."""
    m = float(row.max())
    return float(row[token] - m - np.log(np.exp(row - m).sum()))


def masked_marginals(model, seqs, rows, threshold=1.2, max_batch=256):
    """[n, V]: log-softmax of sequence i's logits at row rows[i], from the
    scheduled forward (eval/proteingym.py:84-98)."""
    lg = forward_scheduled(model, seqs, threshold, max_batch)
    V = model.config.vocab_size
    return np.array([[log_softmax_at(lg[i][r], t) for t in range(V)]
                     for i, r in enumerate(rows)], F32)


# ------------------------------------------------- the compiled reference
class RefModel:
    """esm::Model from the reference compiled in oracle/_ref."""

    def __init__(self, path):
        self.h = ref().ref_model_load(str(path).encode())
        if not self.h:
            raise RuntimeError(ref().ref_last_error().decode())
        cfg = np.zeros(7, np.int32)
        ref_check(ref().ref_model_config(C.c_void_p(self.h), cfg.ctypes.data), "config")
        self.layers, self.d, self.heads, self.dh, self.ffn, self.vocab, self.quantized = map(int, cfg)

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_model_free(C.c_void_p(self.h))
            self.h = None

    def forward_packed(self, ids, cu, masks=None):
        ids, cu = _a(ids, np.int32), _a(cu, np.int32)
        out = np.zeros((ids.size, self.vocab), F32)
        m = None if masks is None else _a(masks, np.int32)
        ref_check(ref().ref_model_forward_packed(C.c_void_p(self.h), ids.ctypes.data,
                                                 None if m is None else m.ctypes.data,
                                                 C.c_int(ids.size), cu.ctypes.data,
                                                 C.c_int(cu.size - 1), out.ctypes.data), "forward_packed")
        return out

    def forward_hidden(self, ids):
        """Model::ForwardWithHiddenStates for one sequence: (logits [L, V],
        hidden [num_layers + 1, L, d])."""
        ids = _a(ids, np.int32)
        L = ids.size
        logits = np.zeros((L, self.vocab), F32)
        hidden = np.zeros((self.layers + 1, L, self.d), F32)
        ref_check(ref().ref_model_forward_hidden(C.c_void_p(self.h), ids.ctypes.data, C.c_int(L),
                                                 logits.ctypes.data, hidden.ctypes.data),
                  "forward_hidden")
        return logits, hidden

    def forward_scheduled(self, seqs, threshold=1.2, max_batch=256):
        lens = np.array([len(s) for s in seqs], np.int32)
        ids = np.concatenate(seqs).astype(np.int32)
        out = np.zeros((int(lens.sum()), self.vocab), F32)
        ref_check(ref().ref_model_forward_scheduled(C.c_void_p(self.h), ids.ctypes.data,
                                                    lens.ctypes.data, len(seqs), threshold,
                                                    max_batch, out.ctypes.data), "forward_scheduled")
        off = np.concatenate([[0], np.cumsum(lens)])
        return [out[off[i]:off[i + 1]] for i in range(len(seqs))]

    def calibrate_smoothquant(self, seqs, pctile=99.9, alpha=0.5):
        lens = np.array([len(s) for s in seqs], np.int32)
        ids = np.concatenate(seqs).astype(np.int32)
        ref_check(ref().ref_model_calibrate_smoothquant(C.c_void_p(self.h), ids.ctypes.data,
                                                        lens.ctypes.data, len(seqs), pctile, alpha),
                  "calibrate")

    def observe(self, seqs, pctile=99.9):
        """quantize.py calibrate: ForwardWithObserver per sequence, then
        Percentile -> [layers * 4] (sites attn_ln_output, attn_out,
        ffn_ln_output, inter_gelu per layer)."""
        lens = np.array([len(s) for s in seqs], np.int32)
        ids = np.concatenate(seqs).astype(np.int32)
        out = np.zeros(self.layers * 4, F32)
        ref_check(ref().ref_model_observe(C.c_void_p(self.h), ids.ctypes.data, lens.ctypes.data,
                                          len(seqs), C.c_float(pctile), out.ctypes.data), "observe")
        return out

    def apply_smoothquant(self, stats, alpha=0.5):
        """Model::ApplySmoothQuant with stats [layers * 4] as from observe()."""
        st = _a(stats)
        ref_check(ref().ref_model_apply_smoothquant(C.c_void_p(self.h), st.ctypes.data,
                                                    C.c_float(alpha)), "apply_smoothquant")

    def quantize(self):
        ref_check(ref().ref_model_quantize(C.c_void_p(self.h)), "quantize")

    def save_gguf(self, path):
        ref_check(ref().ref_model_save_gguf(C.c_void_p(self.h), str(path).encode()), "save_gguf")


def ref_force_isa(isa: str | None):
    ref().ref_force_isa(isa.encode() if isa else None)
