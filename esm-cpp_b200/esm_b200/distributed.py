"""ForwardScheduled sharded over ranks (one process per GPU, torch.distributed).

The packed groups that PlanBatches makes are independent units: each rank
runs a disjoint subset on its own weight replica and the only cross-device
step is gathering the per-sequence logits to the host of rank 0 (there is no
collective on the forward).  Groups go to ranks longest-processing-time
first on the cost sum_b(24*d^2*L_b + 4*d*L_b^2) -- the same rule as the
in-process multi-device dispatcher (esmcu_forward_scheduled_multi).
"""
from __future__ import annotations

import numpy as np


def group_cost(lengths, d: int) -> float:
    return float(sum(24.0 * d * d * L + 4.0 * d * L * L for L in lengths))


def assign_groups(plan, lengths, world: int, d: int):
    """LPT: groups by descending cost, each to the least-loaded rank (lowest
    rank on ties).  Returns one list of group indices per rank."""
    costs = [(group_cost([lengths[i] for i in g], d), gi) for gi, g in enumerate(plan)]
    costs.sort(key=lambda c: -c[0])
    load = [0.0] * world
    out = [[] for _ in range(world)]
    for c, gi in costs:
        r = min(range(world), key=lambda k: (load[k], k))
        load[r] += c
        out[r].append(gi)
    return out


def forward_scheduled_sharded(run_group, input_ids, rank: int, world: int, d: int,
                              imbalance_threshold: float = 1.2, max_batch_size: int = 256,
                              dst: int = 0, group=None):
    """Runs this rank's share of the plan with run_group(packed_ids, cu) ->
    packed logits [T, V] and gathers every sequence's logits to rank `dst`
    (returned there in input order; other ranks return None)."""
    import torch.distributed as dist

    from .ops import plan_batches

    seqs = [np.ascontiguousarray(s, np.int32) for s in input_ids]
    lens = [int(s.shape[0]) for s in seqs]
    plan = plan_batches(np.array(lens, np.int32), imbalance_threshold, max_batch_size)
    mine = assign_groups(plan, lens, world, d)[rank]
    local = {}
    for gi in mine:
        g = plan[gi]
        ids = np.concatenate([seqs[i] for i in g]) if g else np.zeros(0, np.int32)
        cu = np.concatenate([[0], np.cumsum([lens[i] for i in g])]).astype(np.int32)
        logits = run_group(ids, cu)
        for j, i in enumerate(g):
            local[i] = np.ascontiguousarray(logits[cu[j]:cu[j + 1]])
    gathered = [None] * world if rank == dst else None
    dist.gather_object(local, gathered, dst=dst, group=group)
    if rank != dst:
        return None
    merged = {}
    for part in gathered:
        merged.update(part)
    return [merged[i] for i in range(len(seqs))]
