"""Small, self-checking cases of the hot kernels, sized for a profiler capture.

    python kernel_cases.py layer|gemm|ln|attn|attn_long|attn_time|all

Each case holds a few hundred MB on the device at most (inputs still larger
than L2 where the kernel streams them) and launches its kernel a handful of
times, so `ncu -k regex:<kernel> -s <n> -c <k>` over it ends in a minute or two.

  layer  one group of the bench workload (ESM-2-650M width, 2 layers, SmoothQuant
         W8A8, the first PlanBatches group of the rank-0 sequences) through
         forward_packed: every kernel of the forward at its production shape
  gemm   linear_int8 at the fc1/QKV shape M=16384, N=3840, K=1280
  ln     layernorm over 32768 x 1280
  attn   attention_varlen over 512 sequences of the bench length distribution
         (20 heads, head_dim 64)
  attn_long  attention_varlen over 128 sequences of 402 tokens (the
         deep-mutational-scan length; the > 256 kernel), 20 heads, head_dim 64
  attn_time  CUDA-event timing of attention_varlen at equal-length shapes
         (10 launches after 3 warm-ups each), one JSON line; not for ncu
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent / "esm-cpp_b200"))

from esm_b200 import ops, synth  # noqa: E402


def _layer():
    m = synth.quantized_650m(seed=0, num_layers=2)
    lens = synth.varlen_lengths(256, seed=1000)
    seqs = synth.residue_ids(lens, seed=2000)
    plan = ops.plan_batches([len(s) for s in seqs], 1.2, 256)
    group = [seqs[i] for i in plan[0]]
    ids, cu = synth.pack(group)
    out = np.empty((ids.size, m.config.vocab_size), np.float32)
    for _ in range(3):
        m.forward_packed(ids, cu, out=out)
    assert np.isfinite(out).all()
    print(f"layer ok: {len(group)} sequences, {ids.size} tokens")
    m.close()


def _gemm(torch, dev):
    M, N, K = 16384, 3840, 1280
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn((M, K), device=dev, generator=g)
    Wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
    ws = torch.full((N,), 1e-3, device=dev)
    b = torch.zeros(N, device=dev)
    for _ in range(3):
        C = ops.linear_int8(A, Wq, ws, b)
    ops.synchronize()
    assert bool(torch.isfinite(C).all())
    print("gemm ok", float(C.abs().max()))


def _ln(torch, dev):
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn((32768, 1280), device=dev, generator=g)
    gamma, beta = torch.ones(1280, device=dev), torch.zeros(1280, device=dev)
    for _ in range(3):
        y = ops.layernorm(x, gamma, beta)
    ops.synchronize()
    assert bool(torch.isfinite(y).all())
    print("ln ok", float(y.abs().max()))


def _attn(torch, dev):
    lens = synth.varlen_lengths(512, seed=3) + 2
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev)
    T, H, dh = int(cu[-1]), 20, 64
    g = torch.Generator(device=dev).manual_seed(2)
    q = torch.randn((T, H, dh), device=dev, generator=g) * 0.125
    k = torch.randn((T, H, dh), device=dev, generator=g)
    v = torch.randn((T, H, dh), device=dev, generator=g)
    for _ in range(2):
        o = ops.attention_varlen(q, k, v, cu, H, dh)
    ops.synchronize()
    assert bool(torch.isfinite(o).all())
    print("attn ok", T, float(o.abs().max()))


def _attn_long(torch, dev):
    lens = np.full(128, 402, np.int64)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev)
    T, H, dh = int(cu[-1]), 20, 64
    g = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn((T, H, dh), device=dev, generator=g) * 0.125
    k = torch.randn((T, H, dh), device=dev, generator=g)
    v = torch.randn((T, H, dh), device=dev, generator=g)
    for _ in range(2):
        o = ops.attention_varlen(q, k, v, cu, H, dh)
    ops.synchronize()
    assert bool(torch.isfinite(o).all())
    print("attn_long ok", T, float(o.abs().max()))


def _attn_time(torch, dev):
    import json

    res = {}
    for nseq, L in ((512, 122), (256, 250), (400, 402), (128, 402), (256, 300), (64, 1000)):
        cu = torch.tensor(np.arange(nseq + 1, dtype=np.int32) * L, device=dev)
        T, H, dh = nseq * L, 20, 64
        g = torch.Generator(device=dev).manual_seed(4)
        q = torch.randn((T, H, dh), device=dev, generator=g) * 0.125
        k = torch.randn((T, H, dh), device=dev, generator=g)
        v = torch.randn((T, H, dh), device=dev, generator=g)
        for _ in range(3):
            ops.attention_varlen(q, k, v, cu, H, dh)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            ops.attention_varlen(q, k, v, cu, H, dh)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 10
        res[f"{nseq}x{L}"] = {"ms": round(ms, 3),
                              "tflops": round(nseq * H * L * L * dh * 4 / ms / 1e9, 1)}
        del q, k, v
    print(json.dumps(res))


def main(argv=None) -> int:
    import torch

    which = (argv if argv is not None else sys.argv[1:]) or ["all"]
    which = which[0]
    dev = torch.device("cuda:0")
    if which in ("layer", "all"):
        _layer()
    if which in ("gemm", "all"):
        _gemm(torch, dev)
    if which in ("ln", "all"):
        _ln(torch, dev)
    if which in ("attn", "all"):
        _attn(torch, dev)
    if which in ("attn_long", "all"):
        _attn_long(torch, dev)
    if which == "attn_time":
        _attn_time(torch, dev)
    return 0


if __name__ == "__main__":
    sys.exit(main())
