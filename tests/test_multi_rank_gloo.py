"""The N > 1 path on the CPU: world_size-2 gloo ranks shard ForwardScheduled
by packed group and gather logits to rank 0.  The per-group compute is the
CPU oracle (a tiny model), so only the sharding / gathering / reordering
logic is under test; the GPU per-group path is covered by the -m gpu tests.
A rank that fails makes the others fail on the host (short process-group
timeout), never hang."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
TINY = dict(num_hidden_layers=1, hidden_size=64, num_attention_heads=1, head_dim=64,
            intermediate_size=128)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _workload():
    from esm_b200 import synth

    return synth.residue_ids(synth.varlen_lengths(23, seed=3, mean=40, sd=25, lo=1, hi=90), seed=4)


def _worker(rank, world, port, outdir, fail_rank, max_batch=5, threshold=1.2):
    import datetime

    for p in (str(ROOT / "esm-cpp_b200"), str(ROOT / "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    import oracle as O
    from esm_b200 import synth
    from esm_b200.distributed import forward_scheduled_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        m = synth.random_model(TINY, seed=9)
        m.quantize_weights()

        def run_group(ids, cu):
            if rank == fail_rank:
                raise RuntimeError("injected failure on rank %d" % rank)
            return O.forward_packed(m, ids, cu)

        try:
            out = forward_scheduled_sharded(run_group, _workload(), rank, world, d=64,
                                            imbalance_threshold=threshold,
                                            max_batch_size=max_batch)
            status = "ok"
        except Exception as e:  # noqa: BLE001
            out, status = None, f"error: {type(e).__name__}"
        if rank == 0 and out is not None:
            np.savez(Path(outdir) / "out.npz", *out)
        (Path(outdir) / f"status{rank}.txt").write_text(status)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _spawn(tmp_path, fail_rank=-1, world=2, max_batch=5, threshold=1.2):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(world, _port(), str(tmp_path), fail_rank, max_batch, threshold),
                       nprocs=world, join=True, start_method="spawn")


@pytest.mark.parametrize("world,max_batch,threshold", [(2, 5, 1.2), (3, 12, 1000.0)])
def test_sharded_scheduled_forward_equals_single_process(tmp_path, O, world, max_batch, threshold):
    """(3, 12, no split): 23 sequences make two groups, so rank 2 runs none
    and sends only padding; the two others hold different token counts."""
    from esm_b200 import synth
    from esm_b200.distributed import plan_shards

    _spawn(tmp_path, world=world, max_batch=max_batch, threshold=threshold)
    for r in range(world):
        assert (tmp_path / f"status{r}.txt").read_text() == "ok"
    sp = plan_shards([len(s) for s in _workload()], world, 64, threshold, max_batch)
    if world == 3:
        assert sorted(len(a) for a in sp.assign) == [0, 1, 1]
        assert len(set(sp.tokens)) == 3
    got = np.load(tmp_path / "out.npz")
    seqs = _workload()
    m = synth.random_model(TINY, seed=9)
    m.quantize_weights()
    from esm_b200.ops import plan_batches

    lens = [len(s) for s in seqs]
    for g in plan_batches(np.array(lens, np.int32), threshold, max_batch):  # same groups, same numerics
        ids = np.concatenate([seqs[i] for i in g])
        cu = np.concatenate([[0], np.cumsum([lens[i] for i in g])]).astype(np.int32)
        want = O.forward_packed(m, ids, cu)
        for j, i in enumerate(g):
            assert np.array_equal(got[f"arr_{i}"], want[cu[j]:cu[j + 1]])


def test_failing_rank_is_reported_not_hung(tmp_path):
    _spawn(tmp_path, fail_rank=1)
    assert (tmp_path / "status1.txt").read_text().startswith("error")
    assert (tmp_path / "status0.txt").read_text().startswith("error")


def test_lpt_assignment_balances_and_covers():
    from esm_b200.distributed import assign_groups, group_cost

    rng = np.random.default_rng(0)
    lens = rng.integers(50, 400, 64).tolist()
    plan = [list(range(i, min(i + 4, 64))) for i in range(0, 64, 4)]
    for world in (1, 2, 4, 8):
        a = assign_groups(plan, lens, world, 1280)
        assert sorted(sum(a, [])) == list(range(len(plan)))
        loads = [sum(group_cost([lens[i] for i in plan[g]], 1280) for g in r) for r in a]
        biggest = max(group_cost([lens[i] for i in g], 1280) for g in plan)
        assert max(loads) - min(loads) <= biggest


def test_dms_sharding_gives_every_gpu_equal_groups():
    """Config 4: 7,601 sequences of 402 tokens, groups of at most 256; the
    bench's max_batch rule makes the group count a multiple of the GPU count,
    so LPT gives every GPU the same number of groups and tokens within one
    group's worth."""
    import importlib.util

    from esm_b200.distributed import plan_shards

    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    lens = [402] * 7601
    for world in (1, 2, 4, 8):
        mb = bench._dms_max_batch(len(lens), world)
        assert mb <= 256
        sp = plan_shards(lens, world, 2560, 1.2, mb)
        counts = [len(a) for a in sp.assign]
        assert len(sp.plan) % world == 0 and len(set(counts)) == 1, (world, counts)
        assert max(sp.tokens) - min(sp.tokens) <= mb * 402
        assert sp.imbalance < 1.01
