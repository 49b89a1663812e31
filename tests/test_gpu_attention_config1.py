"""BASELINE config 1 at full size: the isolated varlen attention op at 650M
shape, 4096 sequences with lengths ~ Normal(120, 30) clipped to [90, 250]
(about 490k packed tokens), 20 heads x 64, Q/K/V drawn N(0, 1).  The op is
the reference's sequence inside TransformerBlock (model.cpp:976-988):
Q *= 1/sqrt(64), RoPE (base 10000) on Q and K with positions restarting per
sequence, then AttentionVarlen.  Inputs and output take about 10 GB of HBM.

Every output row must be finite, and 24 sequences spread over the batch
(all 20 heads, the shortest and the longest included) are recomputed by the
oracle from the same inputs: FP32 within 1e-4 * (1 + |ref|), and with
ESM_AMX_ATTENTION=on (the reference's BF16 attention) within the same class
of the oracle's BF16 form.  Attention is per sequence, so checking a
sequence alone checks it inside the full batch.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, DH = 20, 64


@pytest.fixture(scope="module")
def config1(cuda):
    import torch

    from esm_b200 import ops, synth

    lens = synth.varlen_lengths(4096, seed=101)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    g = torch.Generator(device=cuda).manual_seed(102)
    qkv = torch.randn((3, T, H, DH), generator=g, device=cuda, dtype=torch.float32)
    cos_t, sin_t = ops.rope_build_tables(int(lens.max()), DH)
    dcos, dsin = torch.from_numpy(cos_t).to(cuda), torch.from_numpy(sin_t).to(cuda)
    dcu = torch.from_numpy(cu).to(cuda)
    pick = sorted(set([int(np.argmin(lens)), int(np.argmax(lens))] +
                      list(np.linspace(0, 4095, 22).astype(int))))
    # Host copies of the picked sequences' raw inputs, for the oracle.
    raw = {b: qkv[:, cu[b]:cu[b + 1]].cpu().numpy() for b in pick}
    q, k, v = qkv[0], qkv[1], qkv[2]
    ops.scale_inplace(q, 1.0 / 8.0)
    ops.rope_apply_varlen(q, dcos, dsin, dcu, H, DH)
    ops.rope_apply_varlen(k, dcos, dsin, dcu, H, DH)
    yield dict(lens=lens, cu=cu, T=T, q=q, k=k, v=v, dcu=dcu, pick=pick, raw=raw,
               cos=cos_t, sin=sin_t)
    del qkv


def _oracle(O, c, b, bf16):
    q, k, v = (np.ascontiguousarray(x) for x in c["raw"][b])
    L = q.shape[0]
    cu1 = np.array([0, L], np.int32)
    q = (q * np.float32(1.0 / 8.0)).astype(np.float32)
    q = O.rope_apply_varlen(q, c["cos"], c["sin"], cu1, H, DH)
    k = O.rope_apply_varlen(k, c["cos"], c["sin"], cu1, H, DH)
    return O.attention_varlen(q, k, v, cu1, H, DH, bf16=bf16)


@pytest.mark.parametrize("bf16", [False, True])
def test_config1_full_size_attention(config1, O, monkeypatch, record, bf16):
    from esm_b200 import ops

    c = config1
    if bf16:
        monkeypatch.setenv("ESM_AMX_ATTENTION", "on")
    else:
        monkeypatch.delenv("ESM_AMX_ATTENTION", raising=False)
    assert 450_000 < c["T"] < 530_000
    out = ops.attention_varlen(c["q"], c["k"], c["v"], c["dcu"], H, DH)
    ops.synchronize()
    assert bool(out.isfinite().all())
    worst = 0.0
    for b in c["pick"]:
        got = out[c["cu"][b]:c["cu"][b + 1]].cpu().numpy()
        want = _oracle(O, c, b, bf16)
        err = float((np.abs(got - want) / (1.0 + np.abs(want))).max())
        worst = max(worst, err)
    record("config1_attention_" + ("bf16" if bf16 else "fp32"), tokens=c["T"],
           sequences_checked=len(c["pick"]), max_rel_err=worst)
    assert worst <= 1e-4, worst
