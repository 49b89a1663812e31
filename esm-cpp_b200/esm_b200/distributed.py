"""ForwardScheduled sharded over ranks (one process per GPU, torch.distributed).

The packed groups that PlanBatches makes (sched/scheduler.cpp:54-75) are
independent units: each rank runs a disjoint subset on its own weight replica
and the only cross-device step is gathering the logits to rank `dst` (there
is no collective on the forward).  Groups go to ranks longest-processing-time
first on the cost sum_b(24*d^2*L_b + 4*d*L_b^2) -- the same rule as the
in-process multi-device dispatcher (esmcu_forward_scheduled_multi).

The gather is one `torch.distributed.gather` of each rank's packed logits
[T_rank, V] (padded to the largest rank's T): over NCCL (NVLink) for CUDA
tensors, over gloo for CPU tensors.  Rank `dst` then reorders the rows into
per-sequence outputs in caller order.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def group_cost(lengths, d: int) -> float:
    return float(sum(24.0 * d * d * L + 4.0 * d * L * L for L in lengths))


def assign_groups(plan, lengths, world: int, d: int):
    """LPT: groups by descending cost (lower group index first on ties),
    each to the least-loaded rank (lowest rank on ties).  Returns one list of
    group indices per rank, deterministic on every rank."""
    costs = [(group_cost([lengths[i] for i in g], d), gi) for gi, g in enumerate(plan)]
    costs.sort(key=lambda c: (-c[0], c[1]))
    load = [0.0] * world
    out = [[] for _ in range(world)]
    for c, gi in costs:
        r = min(range(world), key=lambda k: (load[k], k))
        load[r] += c
        out[r].append(gi)
    return out


@dataclass
class ShardPlan:
    """PlanBatches groups, their LPT assignment and each rank's packed rows:
    rank r runs groups assign[r] in order, its packed logits hold those
    groups' sequences back to back (tokens[r] rows)."""
    lens: list
    plan: list
    assign: list
    tokens: list
    loads: list

    @property
    def max_tokens(self) -> int:
        return max(self.tokens) if self.tokens else 0

    @property
    def imbalance(self) -> float:
        """Largest rank cost over the mean rank cost (1.0 = perfect)."""
        mean = sum(self.loads) / max(len(self.loads), 1)
        return max(self.loads) / mean if mean > 0 else 1.0

    def rank_sequences(self, r: int):
        """(sequence index, packed row offset) of rank r's sequences."""
        out, off = [], 0
        for gi in self.assign[r]:
            for i in self.plan[gi]:
                out.append((i, off))
                off += self.lens[i]
        return out


def plan_shards(lens, world: int, d: int, imbalance_threshold: float = 1.2,
                max_batch_size: int = 256) -> ShardPlan:
    from .ops import plan_batches

    lens = [int(x) for x in lens]
    plan = plan_batches(np.array(lens, np.int32), imbalance_threshold, max_batch_size)
    assign = assign_groups(plan, lens, world, d)
    tokens = [sum(lens[i] for gi in a for i in plan[gi]) for a in assign]
    loads = [sum(group_cost([lens[i] for i in plan[gi]], d) for gi in a) for a in assign]
    return ShardPlan(lens, plan, assign, tokens, loads)


def pack_group(seqs, plan, gi, lens):
    g = plan[gi]
    ids = np.concatenate([seqs[i] for i in g]).astype(np.int32) if g else np.zeros(0, np.int32)
    cu = np.concatenate([[0], np.cumsum([lens[i] for i in g])]).astype(np.int32)
    return ids, cu


def gather_logits(local, sp: ShardPlan, rank: int, world: int, n_seqs: int, dst: int = 0,
                  group=None):
    """Gathers every rank's packed logits `local` (a torch tensor [>= tokens
    of the rank, V], CUDA for NCCL or CPU for gloo, rows past the rank's
    tokens ignored) to rank `dst` and returns there the per-sequence logits
    (numpy) in input order; other ranks return None."""
    import torch
    import torch.distributed as dist

    V = local.shape[1]
    T = sp.max_tokens
    if local.shape[0] != T:
        pad = torch.zeros((T, V), dtype=local.dtype, device=local.device)
        pad[: min(local.shape[0], T)] = local[:T]
        local = pad
    bufs = [torch.empty_like(local) for _ in range(world)] if rank == dst else None
    dist.gather(local.contiguous(), bufs, dst=dst, group=group)
    if rank != dst:
        return None
    host = [b.cpu().numpy() for b in bufs]
    out = [None] * n_seqs
    for r in range(world):
        for i, off in sp.rank_sequences(r):
            out[i] = host[r][off:off + sp.lens[i]]
    return out


def forward_scheduled_sharded(run_group, input_ids, rank: int, world: int, d: int,
                              imbalance_threshold: float = 1.2, max_batch_size: int = 256,
                              dst: int = 0, group=None, vocab: int = 33, device=None):
    """Runs this rank's share of the plan with run_group(packed_ids, cu) ->
    packed logits [T, V] (numpy, or a torch tensor on `device`) and gathers
    every sequence's logits to rank `dst` (returned there in input order;
    other ranks return None).  device: where the gathered tensors live (a
    CUDA device for NCCL; None = CPU, for gloo)."""
    import torch

    seqs = [np.ascontiguousarray(s, np.int32) for s in input_ids]
    sp = plan_shards([s.shape[0] for s in seqs], world, d, imbalance_threshold, max_batch_size)
    dev = torch.device("cpu") if device is None else torch.device(device)
    local = torch.zeros((max(sp.max_tokens, 1), vocab), dtype=torch.float32, device=dev)
    off = 0
    for gi in sp.assign[rank]:
        ids, cu = pack_group(seqs, sp.plan, gi, sp.lens)
        logits = run_group(ids, cu)
        t = logits if isinstance(logits, torch.Tensor) else torch.from_numpy(np.asarray(logits))
        local[off:off + ids.shape[0]] = t.to(dev)
        off += ids.shape[0]
    if sp.max_tokens == 0:
        return [np.zeros((0, vocab), np.float32) for _ in seqs] if rank == dst else None
    return gather_logits(local, sp, rank, world, len(seqs), dst, group)


class _Staging:
    """Per-device pinned host buffer for the rank's packed ids, reused across
    calls: grown when too small, and rewritten only after the event recorded
    behind the previous call's host-to-device copies has completed."""

    def __init__(self):
        self.buf = None
        self.done = None

    def take(self, n: int, dev):
        import torch

        if self.done is not None:
            self.done.synchronize()
        if self.buf is None or self.buf.numel() < n:
            self.buf = torch.empty(max(n, 1), dtype=torch.int32, pin_memory=True)
        return self.buf

    def mark(self, dev):
        import torch

        self.done = torch.cuda.Event()
        self.done.record(torch.cuda.current_stream(dev))


_staging = {}


def forward_scheduled_sharded_device(model, input_ids, rank: int, world: int,
                                     imbalance_threshold: float = 1.2, max_batch_size: int = 256,
                                     dst: int = 0, group=None):
    """forward_scheduled_sharded on this rank's GPU model (esm_b200.Model):
    the rank's packed ids go to the device through a pinned staging buffer
    (one asynchronous host-to-device copy per group), each group runs on the
    device into one packed logits buffer, and the buffer is gathered to rank
    `dst` over NCCL.  Returns the logits per sequence in input order on rank
    `dst`, None elsewhere."""
    import torch

    seqs = [np.ascontiguousarray(s, np.int32) for s in input_ids]
    sp = plan_shards([s.shape[0] for s in seqs], world, model.config.hidden_size,
                     imbalance_threshold, max_batch_size)
    dev = torch.device("cuda", model.device)
    V = model.config.vocab_size
    local = torch.zeros((max(sp.max_tokens, 1), V), dtype=torch.float32, device=dev)
    st = _staging.setdefault(model.device, _Staging())
    host = st.take(sp.tokens[rank], dev)
    d_ids_all = torch.empty(max(sp.tokens[rank], 1), dtype=torch.int32, device=dev)
    off = 0
    for gi in sp.assign[rank]:
        ids, cu = pack_group(seqs, sp.plan, gi, sp.lens)
        n = ids.shape[0]
        host[off:off + n].numpy()[:] = ids
        d_ids = d_ids_all[off:off + n]
        d_ids.copy_(host[off:off + n], non_blocking=True)
        model.forward_packed_device(d_ids, cu, local[off:off + n])
        off += n
    st.mark(dev)
    if sp.max_tokens == 0:
        return [np.zeros((0, V), np.float32) for _ in seqs] if rank == dst else None
    return gather_logits(local, sp, rank, world, len(seqs), dst, group)
