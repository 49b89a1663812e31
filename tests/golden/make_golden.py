"""Generates tests/golden/*.npz from the reference esm.cpp, compiled from its
own sources into oracle/_ref (make -C oracle ref).  Run in a container that
has the reference sources; the fixtures then travel with the repository and
pin the oracle restatement and the GPU path where the reference is absent.

    python tests/golden/make_golden.py

Every array is produced by a reference entry point named in the key:
  lin8_*     LinearInt8 on the VNNI path (one activation scale over M) and the
             default dispatch, QuantizeActPrefixAvx512 scale + u8 codes.
  attn_*     AttentionVarlenRef and the default AttentionVarlen.
  ln_*       LayerNormRef and LayerNorm; gelu_*: GeluRef and Gelu.
  rope_*     RopeBuildTables, RopeApplyVarlenRef / RopeApplyVarlen.
  plan_*     PlanBatches.
  model_*    Model::ForwardPacked of a tiny W8A8 model (its Q8_ESM GGUF
             tensors are stored alongside) and of the same model in FP32.
  hidden_*   Model::ForwardWithHiddenStates of that model, FP32 and W8A8
             (hidden_golden.npz), one sequence at a time, concatenated.
  optin_golden.npz  the opt-in paths on that model: INT8 LM head, the
             layer-0 fc1 fp16 flag, BF16 attention, masked-marginal
             log-probabilities.
"""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "esm-cpp_b200"))

import oracle as O  # noqa: E402

F32 = np.float32


def ops_fixture(path):
    R = O.ref()
    rng = np.random.default_rng(20261201)
    out = {}
    # W8A8 linear: M with a non-multiple-of-32 tail, N, K multiples of 64
    M, N, K = 45, 128, 256
    A = rng.standard_normal((M, K)).astype(F32)
    A[:, rng.integers(0, K, 3)] *= 20.0
    W = (rng.standard_normal((N, K)) * 0.02).astype(F32)
    q = np.zeros((N, K), np.int8)
    s = np.zeros(N, F32)
    O.ref_check(R.ref_quantize_weights(W.ctypes.data, N, K, q.ctypes.data, s.ctypes.data))
    bias = (rng.standard_normal(N) * 0.1).astype(F32)
    u8 = np.zeros(M * K, np.uint8)
    sc = np.zeros(1, F32)
    O.ref_check(R.ref_quant_act_prefix(A.ctypes.data, A.size, u8.ctypes.data, sc.ctypes.data))
    c_vnni = np.zeros((M, N), F32)
    O.ref_check(R.ref_linear_int8_vnni(A.ctypes.data, q.ctypes.data, s.ctypes.data, bias.ctypes.data,
                                       c_vnni.ctypes.data, M, N, K))
    c_amx = np.zeros((M, N), F32)
    O.ref_check(R.ref_linear_int8_amx(A.ctypes.data, q.ctypes.data, s.ctypes.data, bias.ctypes.data,
                                      c_amx.ctypes.data, M, N, K))
    out.update(lin8_A=A, lin8_W=W, lin8_Wq=q, lin8_ws=s, lin8_bias=bias, lin8_act_u8=u8.reshape(M, K),
               lin8_act_scale=sc, lin8_C_vnni=c_vnni, lin8_C_amx=c_amx)
    # attention
    cu = np.array([0, 1, 18, 18, 83], np.int32)
    H, dh = 4, 64
    T = int(cu[-1])
    qa, ka, va = (rng.standard_normal((3, T, H, dh)).astype(F32))
    qa *= F32(0.125)
    o_ref = np.zeros_like(qa)
    O.ref_check(R.ref_attention_varlen_ref(qa.ctypes.data, ka.ctypes.data, va.ctypes.data, cu.ctypes.data,
                                           len(cu) - 1, H, dh, o_ref.ctypes.data))
    o_def = np.zeros_like(qa)
    O.ref_check(R.ref_attention_varlen(qa.ctypes.data, ka.ctypes.data, va.ctypes.data, cu.ctypes.data,
                                       len(cu) - 1, H, dh, o_def.ctypes.data))
    out.update(attn_cu=cu, attn_q=qa, attn_k=ka, attn_v=va, attn_out_ref=o_ref, attn_out_default=o_def)
    # layernorm / gelu
    x = (rng.standard_normal((6, 1280)) * 2 + 0.3).astype(F32)
    g = rng.standard_normal(1280).astype(F32)
    b = rng.standard_normal(1280).astype(F32)
    y_ref = np.zeros_like(x)
    O.ref_check(R.ref_layernorm_ref(x.ctypes.data, g.ctypes.data, b.ctypes.data, 1e-5, y_ref.ctypes.data, 6, 1280))
    y_def = np.zeros_like(x)
    O.ref_check(R.ref_layernorm(x.ctypes.data, g.ctypes.data, b.ctypes.data, 1e-5, y_def.ctypes.data, 6, 1280))
    xg = (rng.standard_normal(4096) * 4).astype(F32)
    gr = np.zeros_like(xg)
    O.ref_check(R.ref_gelu_ref(xg.ctypes.data, gr.ctypes.data, xg.size))
    gd = np.zeros_like(xg)
    O.ref_check(R.ref_gelu(xg.ctypes.data, gd.ctypes.data, xg.size))
    out.update(ln_x=x, ln_g=g, ln_b=b, ln_out_ref=y_ref, ln_out_default=y_def, gelu_x=xg,
               gelu_out_ref=gr, gelu_out_default=gd)
    # rope
    c = np.zeros((256, 64), F32)
    sn = np.zeros((256, 64), F32)
    O.ref_check(R.ref_rope_build_tables(256, 64, c.ctypes.data, sn.ctypes.data))
    xr = rng.standard_normal((T, H, dh)).astype(F32)
    r_ref = xr.copy()
    O.ref_check(R.ref_rope_apply_varlen_ref(r_ref.ctypes.data, c.ctypes.data, sn.ctypes.data, cu.ctypes.data,
                                            len(cu) - 1, H, dh))
    r_def = xr.copy()
    O.ref_check(R.ref_rope_apply_varlen(r_def.ctypes.data, c.ctypes.data, sn.ctypes.data, cu.ctypes.data,
                                        len(cu) - 1, H, dh))
    out.update(rope_cos=c, rope_sin=sn, rope_x=xr, rope_out_ref=r_ref, rope_out_default=r_def)
    # plan
    lens = rng.integers(5, 300, 300).astype(np.int32)
    order = np.zeros(300, np.int32)
    sizes = np.zeros(300, np.int32)
    ng = R.ref_plan_batches(lens.ctypes.data, 300, 1.2, 64, order.ctypes.data, sizes.ctypes.data)
    out.update(plan_lengths=lens, plan_order=order, plan_sizes=sizes[:ng])
    np.savez_compressed(path, **out)


def model_fixture(path):
    """Tiny ESM-2-shaped model: the reference calibrates, SmoothQuant-
    migrates and quantises it; the fixture stores the Q8_ESM GGUF bytes and
    the reference's packed logits (FP32 and W8A8, VNNI and default ISA)."""
    from esm_b200 import synth

    arch = dict(num_hidden_layers=2, hidden_size=64, num_attention_heads=1, head_dim=64,
                intermediate_size=256)
    m = synth.random_model(arch, seed=77)
    seqs = synth.residue_ids([11, 40, 1, 75], seed=78)
    ids, cu = synth.pack(seqs)
    with tempfile.TemporaryDirectory() as td:
        st = Path(td) / "m.safetensors"
        m.save_to_safetensors(st)
        ref = O.RefModel(st)
        logits_fp32 = ref.forward_packed(ids, cu)
        ref.calibrate_smoothquant(synth.residue_ids([30, 60], seed=79), 99.9, 0.5)
        ref.quantize()
        gg = Path(td) / "m_q8.gguf"
        ref.save_gguf(gg)
        gguf_bytes = np.frombuffer(gg.read_bytes(), np.uint8)
        O.ref_force_isa("avx512vnni")
        logits_vnni = O.RefModel(gg).forward_packed(ids, cu)
        O.ref_force_isa(None)
        logits_default = O.RefModel(gg).forward_packed(ids, cu)
        fp32_bytes = np.frombuffer(st.read_bytes(), np.uint8)
    np.savez_compressed(path, ids=ids, cu=cu, safetensors=fp32_bytes, logits_fp32=logits_fp32,
                        gguf_q8=gguf_bytes, logits_q8_vnni=logits_vnni,
                        logits_q8_default=logits_default)


def hidden_fixture(path, model_path):
    """Model::ForwardWithHiddenStates (model.h:185-191) of the reference on
    the tiny model of `model_fixture`, one sequence at a time: the embedding
    output, each block's output but the last, and the final-LN output, for the
    FP32 model and the W8A8 model (VNNI ISA)."""
    M = np.load(model_path)
    ids, cu = M["ids"], M["cu"]
    out = {}
    with tempfile.TemporaryDirectory() as td:
        st = Path(td) / "m.safetensors"
        st.write_bytes(M["safetensors"].tobytes())
        gg = Path(td) / "m_q8.gguf"
        gg.write_bytes(M["gguf_q8"].tobytes())
        O.ref_force_isa("avx512vnni")
        for tag, p in (("fp32", st), ("q8", gg)):
            ref = O.RefModel(p)
            hs, lg = [], []
            for b in range(len(cu) - 1):
                logits, hidden = ref.forward_hidden(ids[cu[b]:cu[b + 1]])
                hs.append(hidden)
                lg.append(logits)
            out[f"hidden_{tag}"] = np.concatenate(hs, axis=1)
            out[f"logits_{tag}"] = np.concatenate(lg, axis=0)
        O.ref_force_isa(None)
    np.savez_compressed(path, **out)


def bf16_attention_inputs():
    """Seeded q (scaled by 1/8), k, v [T, 2, 64] and cu for the BF16-attention
    fixture: lengths 60, 7, 270, 1."""
    rng = np.random.default_rng(96)
    H, dh = 2, 64
    cu = np.concatenate([[0], np.cumsum([60, 7, 270, 1])]).astype(np.int32)
    q, k, v = rng.standard_normal((3, int(cu[-1]), H, dh)).astype(F32)
    q *= F32(0.125)
    return q, k, v, cu, H, dh


def optin_fixture(path, model_path):
    """The reference's opt-in paths on the tiny model of `model_fixture`:
    ESM_QUANTIZE_LM_HEAD=on logits of its calibrated, migrated model
    (model.cpp:1487-1492, 1209-1211); the
    logits of a GGUF carrying esm.first_block_fc1_fp16 (model.cpp:250-254,
    1031-1033); ESM_AMX_ATTENTION=on attention (attention.cpp:686-700, run in
    a child process: the reference reads the variable once per process); and
    masked-marginal log-probabilities from its ForwardScheduled
    (eval/proteingym.py:75-98).  Logits use the VNNI ISA (one activation
    scale per operand)."""
    import os
    import subprocess

    from esm_b200 import Model, synth

    M = np.load(model_path)
    ids, cu = M["ids"], M["cu"]
    out = {}
    with tempfile.TemporaryDirectory() as td:
        st = Path(td) / "m.safetensors"
        st.write_bytes(M["safetensors"].tobytes())
        # INT8 LM head, on the calibrated + migrated model of model_fixture
        # (same calibration, so the layers equal gguf_q8's and match the
        # oracle to the FP32 class; SmoothQuant leaves lm_head.dense alone)
        ref = O.RefModel(st)
        ref.calibrate_smoothquant(synth.residue_ids([30, 60], seed=79), 99.9, 0.5)
        os.environ["ESM_QUANTIZE_LM_HEAD"] = "on"
        try:
            ref.quantize()
        finally:
            del os.environ["ESM_QUANTIZE_LM_HEAD"]
        O.ref_force_isa("avx512vnni")
        out["lmhead8_logits"] = ref.forward_packed(ids, cu)
        # layer-0 fc1 fp16 flag, travelling in a GGUF this package writes
        m = Model.load(st)
        m.quantize_weights()
        m.set_first_block_fc1_fp16(True)
        gg = Path(td) / "fc1.gguf"
        m.save_to_gguf(gg)
        out["fc1fp16_gguf"] = np.frombuffer(gg.read_bytes(), np.uint8)
        out["fc1fp16_logits"] = O.RefModel(gg).forward_packed(ids, cu)
        # masked marginals: one masked copy of a wild type per position
        wt = synth.residue_ids([40], seed=95)[0]
        pos = np.array([0, 7, 19, 39], np.int32)
        copies = []
        for p in pos:
            x = wt.copy()
            x[p + 1] = 32
            copies.append(x)
        lg = O.RefModel(st).forward_scheduled(copies)
        out["mm_wt"], out["mm_pos"] = wt, pos
        out["mm_logprobs"] = np.array([[O.log_softmax_at(lg[i][p + 1], t) for t in range(33)]
                                       for i, p in enumerate(pos)], F32)
        O.ref_force_isa(None)
        # BF16 attention, in a child process with the variable set; the
        # inputs are regenerated from the seed by the test (their sums are
        # stored to catch a change of the generator's stream)
        q, k, v, acu, H, dh = bf16_attention_inputs()
        np.savez(Path(td) / "att.npz", q=q, k=k, v=v, cu=acu)
        script = (
            "import sys, numpy as np\n"
            f"sys.path.insert(0, {str(ROOT / 'oracle')!r})\n"
            "import oracle as O\n"
            f"d = np.load({str(Path(td) / 'att.npz')!r})\n"
            "q, k, v, cu = (np.ascontiguousarray(d[n]) for n in ('q', 'k', 'v', 'cu'))\n"
            "o = np.zeros_like(q)\n"
            f"O.ref_check(O.ref().ref_attention_varlen(q.ctypes.data, k.ctypes.data, v.ctypes.data, "
            f"cu.ctypes.data, cu.size - 1, {H}, {dh}, o.ctypes.data))\n"
            f"np.save({str(Path(td) / 'att_out.npy')!r}, o)\n")
        subprocess.run([sys.executable, "-c", script], check=True,
                       env=dict(os.environ, ESM_AMX_ATTENTION="on"))
        out.update(bf16att_sums=np.array([q.sum(dtype=np.float64), k.sum(dtype=np.float64),
                                          v.sum(dtype=np.float64)]),
                   bf16att_out=np.load(Path(td) / "att_out.npy"))
    np.savez_compressed(path, **out)


if __name__ == "__main__":
    O.build()
    ops_fixture(HERE / "ops_golden.npz")
    model_fixture(HERE / "model_golden.npz")
    hidden_fixture(HERE / "hidden_golden.npz", HERE / "model_golden.npz")
    optin_fixture(HERE / "optin_golden.npz", HERE / "model_golden.npz")
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size, "bytes")
