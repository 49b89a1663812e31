"""Headline benchmark: packed residues/s of the ESM-2 650M W8A8 varlen packed
forward (BASELINE config 3a) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step = ForwardScheduled over 256 synthetic sequences (residues ~ N(120,30)
clipped to [90,250], + CLS/EOS; seed per rank) on random-init 650M weights
(N(0,0.02), LN gamma 1 / beta 0) calibrated on the GPU (99.9th percentile),
SmoothQuant-migrated (alpha 0.5) and quantised to per-channel int8.  With N
GPUs (torchrun, one process per GPU) every rank runs its own 256 sequences on
its own weight replica: weak scaling, no collective on the data path.

  value  device-resident: inputs already in HBM, CUDA events on the model's
         stream around each step, L2 flushed between steps (256 MB write;
         the 0.8 GB of int8 weights streamed per step also exceed L2);
         aggregate over ranks = sum of residues / max over ranks of the time.
  e2e    the public API Model.forward_scheduled with host arrays in (pinned)
         and host logits out, same events on the same stream.
  roofline  the INT8 GEMM family (tcgen05 kernels), algorithmic 2*M*N*K ops per
         launch over their CUDA-event time inside the timed steps.
  cpu_baseline  the reference esm.cpp (compiled from its sources into
         oracle/_ref) on a bounded sample of the same workload, rank 0, N=1.

--impl reference times that reference CPU path alone (rank 0; other ranks
exit 0) on a bounded sample per step, through its own API.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "esm-cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "residues/sec, ESM-2-650M W8A8 varlen packed forward at 1/2/4/8 B200"
N_SEQS = 256
CPU_SAMPLE_SEQS = 12


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _workload(rank: int):
    from esm_b200 import synth

    lens = synth.varlen_lengths(N_SEQS, seed=1000 + rank)
    return synth.residue_ids(lens, seed=2000 + rank)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"esm_b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1].split()[0]))
                mx = float(f[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(device: int, seed: int = 0):
    from esm_b200 import synth

    t0 = time.time()
    m = synth.quantized_650m(seed=seed, device=device)
    m._ensure_device()
    return m, time.time() - t0


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the four INT8
# GEMM launches of one layer, per token: ncu capture of the layer case of
# kernel_cases.py (first config-3a group, 13,305 tokens; QKV 176.4 MB,
# out-proj 97.0 MB, fc1 247.7 MB, fc2 253.2 MB).  Traffic grows with the
# tokens of a launch (activations and outputs; the weights are ~3% of it).
GEMM_DRAM_BYTES_PER_TOKEN_LAYER = 774.30e6 / 13305


def gemm_ops_per_step(groups_T, cfg) -> float:
    d, f, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers
    per_token = 2.0 * L * (d * 3 * d + d * d + d * f + f * d)  # = 24 d^2 L for f = 4d
    return per_token * sum(groups_T)


def run_ours(args, rank: int, world: int, local_rank: int, dist):
    import ctypes as C

    import torch

    from esm_b200 import _lib, ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    model, init_s = build_model(local_rank)
    cfg = model.config
    seqs = _workload(rank)
    lens = np.array([len(s) for s in seqs], np.int32)
    tokens = int(lens.sum())

    # Pre-plan and pre-pack the groups (the host part of ForwardScheduled) and
    # place the inputs in HBM for the device-resident measurement.
    plan = ops.plan_batches(lens, 1.2, 256)
    groups = []
    for g in plan:
        ids = np.concatenate([seqs[i] for i in g]).astype(np.int32)
        cu = np.concatenate([[0], np.cumsum(lens[g])]).astype(np.int32)
        d_ids = torch.from_numpy(ids).to(dev)
        d_logits = torch.empty((ids.size, cfg.vocab_size), dtype=torch.float32, device=dev)
        groups.append((d_ids, cu, d_logits))
    L = _lib.lib()
    stream = torch.cuda.ExternalStream(L.esmcu_get_stream(model._ctx), device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step_device():
        n = 0
        for d_ids, cu, d_logits in groups:
            _lib.call("esmcu_model_forward_packed_device", model._dev, C.c_void_p(d_ids.data_ptr()),
                      None, int(d_ids.numel()), cu.ctypes.data, int(cu.size - 1),
                      C.c_void_p(d_logits.data_ptr()))
            n += L.esmcu_model_last_launch_count(model._dev)
        return n

    def timed(fn, k, profile=False):
        ms, launches = [], 0
        if profile:
            model.set_profiling(True)
        for _ in range(k):
            with torch.cuda.stream(stream):
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launches += fn() or 0
            e1.record(stream)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        prof = model.profile() if profile else None
        if profile:
            model.set_profiling(False)
        return ms, launches, prof

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- warmup, then K device-resident steps
    for _ in range(args.warmup):
        step_device()
    _lib.call("esmcu_synchronize", model._ctx)
    barrier()
    with ClockSampler(local_rank) as clk:
        dev_ms, launches, _ = timed(step_device, args.steps)
        barrier()
    clocks = clk.summary()
    _lib.call("esmcu_synchronize", model._ctx)
    # Per-section times from one more, untimed step with the model's
    # section events on (the events would otherwise sit inside the timed steps).
    _, _, prof = timed(step_device, 1, profile=True)
    _lib.call("esmcu_synchronize", model._ctx)

    # ---- e2e through the public API (host ids in, host logits out)
    pinned_seqs = [torch.from_numpy(s).pin_memory().numpy() for s in seqs]
    for _ in range(max(1, args.warmup)):
        model.forward_scheduled(pinned_seqs)
    barrier()
    e2e_ms, _, _ = timed(lambda: model.forward_scheduled(pinned_seqs) and 0, args.steps)
    barrier()

    step_ms = sum(dev_ms) / len(dev_ms)
    e2e_step_ms = sum(e2e_ms) / len(e2e_ms)
    vals = torch.tensor([step_ms, e2e_step_ms, float(tokens)], dtype=torch.float64, device=dev)
    if dist is not None:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        step_ms_max, e2e_ms_max, tok_sum = float(mx[0]), float(mx[1]), float(sm[2])
    else:
        step_ms_max, e2e_ms_max, tok_sum = step_ms, e2e_step_ms, float(tokens)

    if rank != 0:
        return None

    peaks, peak_kind = _peaks()
    gemm_sections = ("qkv_proj", "attn_out_proj", "fc1", "fc2")
    gemm_ms = sum(prof.get(k, 0.0) for k in gemm_sections)  # one profiled step
    ops_step = gemm_ops_per_step([int(g[0].numel()) for g in groups], cfg)
    achieved = ops_step / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else 0.0
    int8_peak = 2.0 * float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
    sections = {k: round(v, 4) for k, v in sorted(prof.items(), key=lambda kv: -kv[1])}

    out = {
        "metric": METRIC,
        "value": round(tok_sum / (step_ms_max * 1e-3), 1),
        "unit": "residues/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms_max, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "esm2_650m_w8a8_varlen (BASELINE config 3a)",
                   "seqs_per_gpu": N_SEQS, "tokens_per_gpu": tokens, "groups": len(groups),
                   "act_quant": "per_tensor", "parallelism": f"replicas x{world}",
                   "l2": "flushed between steps (256 MB write); 0.8 GB int8 weights per step > L2"},
        "e2e": {"value": round(tok_sum / (e2e_ms_max * 1e-3), 1), "unit": "residues/s",
                "h2d_bytes_per_step": int(sum(4 * s.size for s in seqs) + 4 * (len(seqs) + len(plan))),
                "d2h_bytes_per_step": int(tokens * cfg.vocab_size * 4)},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "gemm_i8 (tcgen05 kind::i8; QKV/out/fc1/fc2)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOP/s",
                     "frac": round(achieved / int8_peak, 4),
                     "peak_source": f"2 x bf16_tflops_sustained ({peak_kind}); dense INT8 = 2 x dense BF16",
                     "traffic": round(GEMM_DRAM_BYTES_PER_TOKEN_LAYER * tokens / (4 * len(groups))),
                     "traffic_unit": "bytes per launch (mean over the step's GEMM launches)",
                     "traffic_source": "ncu capture of the first config-3a group, scaled by tokens"},
        "sections_ms_per_step": sections,
        "init_s": round(init_s, 1),
    }
    if clocks is not None:
        out["clocks"] = clocks
    if world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline(model, seqs)
        except Exception as e:  # the baseline is reported, never required
            out["cpu_baseline"] = {"unavailable": str(e)[:200]}
    return out


def _ref_threads():
    n = os.cpu_count() or 1
    os.environ.setdefault("ESM_NUM_THREADS", str(n))
    return int(os.environ["ESM_NUM_THREADS"])


def cpu_baseline(model, seqs):
    """The reference's ForwardScheduled on a bounded sample of the same
    workload, same quantised weights (via GGUF), all host threads."""
    threads = _ref_threads()
    import oracle as O

    if not O.ref_available():
        return {"unavailable": "oracle/_ref not built"}
    sample = seqs[:CPU_SAMPLE_SEQS]
    toks = sum(len(s) for s in sample)
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "w.gguf"
        model.save_to_gguf(p)
        ref = O.RefModel(p)
    ref.forward_scheduled(sample[:2])
    times = []
    t_end = time.time() + 20.0
    while len(times) < 3 and (not times or time.time() < t_end):
        t0 = time.perf_counter()
        ref.forward_scheduled(sample)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(toks / t, 1), "unit": "residues/s", "cores": threads, "kind": "reference",
            "isa": O.ref().ref_current_isa().decode(),
            "sample": f"{len(sample)} of the {N_SEQS} sequences ({toks} tokens), ForwardScheduled, "
                      f"median of {len(times)}"}


def run_reference(args, rank: int):
    """The reference esm.cpp CPU path alone: random-init FP32 safetensors ->
    its own calibration (ForwardWithObserver, 99.9th pct) -> ApplySmoothQuant
    -> QuantizeWeights, then ForwardScheduled on a bounded sample per step."""
    if rank != 0:
        return None
    threads = _ref_threads()
    import oracle as O
    from esm_b200 import synth

    if not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref (reference built from source) missing"}
    m = synth.random_model("esm2_650m", seed=0)
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "w.safetensors"
        m.save_to_safetensors(p)
        del m
        ref = O.RefModel(p)
    ref.calibrate_smoothquant(synth.residue_ids(synth.varlen_lengths(4, seed=1), seed=2), 99.9, 0.5)
    ref.quantize()
    seqs = _workload(0)
    sample = seqs[:CPU_SAMPLE_SEQS]
    toks = sum(len(s) for s in sample)
    for _ in range(args.warmup):
        ref.forward_scheduled(sample[:2])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.forward_scheduled(sample)
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    v = round(toks / t, 1)
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "residues/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "esm2_650m_w8a8_varlen (BASELINE config 3a)",
                       "sample_seqs_per_step": len(sample), "tokens_per_step": toks},
            "cpu_baseline": {"value": v, "unit": "residues/s", "cores": threads, "kind": "reference",
                             "isa": O.ref().ref_current_isa().decode(),
                             "sample": f"{len(sample)} sequences ({toks} tokens) per step"},
            "e2e": {"value": v, "unit": "residues/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return 0

    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as td

        torch.cuda.set_device(local_rank)
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                              device_id=torch.device("cuda", local_rank))
        dist = td
    try:
        out = run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
