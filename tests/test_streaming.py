"""StreamingScheduler (esm_b200.streaming) host logic on CPU, with fake models
that stand in for Model.forward_scheduled."""
import threading
import time

import numpy as np
import pytest

V = 5


def _logits(ids, mask=None):
    """Deterministic fake logits of one sequence: [L, V]."""
    x = ids.astype(np.float32)[:, None] * np.arange(1, V + 1, dtype=np.float32)
    if mask is not None:
        x = x + 1000.0 * (1 - mask.astype(np.float32))[:, None]
    return x


class FakeModel:
    def __init__(self, delay=0.0, fail_marker=None):
        self.delay, self.fail_marker = delay, fail_marker
        self.batches = []
        self.lock = threading.Lock()

    def forward_scheduled(self, input_ids, attention_masks=None, imbalance_threshold=1.2,
                          max_batch_size=256):
        with self.lock:
            self.batches.append([len(s) for s in input_ids])
        if self.delay:
            time.sleep(self.delay)
        if self.fail_marker is not None and any((s == self.fail_marker).any() for s in input_ids):
            raise RuntimeError("planted failure")
        masks = attention_masks or [None] * len(input_ids)
        return [_logits(s, m) for s, m in zip(input_ids, masks)]


def _seqs(n, seed, lo=3, hi=60):
    rng = np.random.default_rng(seed)
    return [rng.integers(4, 24, int(rng.integers(lo, hi))).astype(np.int32) for _ in range(n)]


def test_results_match_requests_and_batches_respect_the_budget():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel()
    seqs = _seqs(80, 1)
    with StreamingScheduler([m], max_tokens=200, max_wait_ms=20) as s:
        futs = s.submit_many(seqs)
        for f, x in zip(futs, seqs):
            assert np.array_equal(f.result(timeout=10), _logits(x))
    assert sum(len(b) for b in m.batches) == len(seqs)
    for b in m.batches:
        assert sum(b) <= 200 or len(b) == 1


def test_concurrent_callers():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel(delay=0.001)
    errors = []

    def caller(seed, s):
        try:
            seqs = _seqs(30, seed)
            futs = [s.submit(x) for x in seqs]
            for f, x in zip(futs, seqs):
                assert np.array_equal(f.result(timeout=10), _logits(x))
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    with StreamingScheduler([m], max_tokens=500, max_wait_ms=2) as s:
        ts = [threading.Thread(target=caller, args=(i, s)) for i in range(4)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    assert not errors
    assert sum(len(b) for b in m.batches) == 120


def test_work_spreads_over_models():
    from esm_b200.streaming import StreamingScheduler

    a, b = FakeModel(delay=0.02), FakeModel(delay=0.02)
    seqs = _seqs(40, 2)
    with StreamingScheduler([a, b], max_tokens=100, max_wait_ms=1) as s:
        for f, x in zip(s.submit_many(seqs), seqs):
            assert np.array_equal(f.result(timeout=10), _logits(x))
    assert a.batches and b.batches


def test_a_lone_request_waits_at_most_max_wait():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel()
    with StreamingScheduler([m], max_tokens=10**6, max_wait_ms=30) as s:
        t0 = time.monotonic()
        f = s.submit(np.array([5, 6, 7], np.int32))
        f.result(timeout=5)
        assert time.monotonic() - t0 < 2.0
    assert m.batches == [[3]]


def test_failures_reach_their_batch_only():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel(fail_marker=23)
    with StreamingScheduler([m], max_tokens=10**6, max_wait_ms=5) as s:
        bad = s.submit(np.array([4, 23, 5], np.int32))
        with pytest.raises(RuntimeError, match="planted failure"):
            bad.result(timeout=5)
        good = s.submit(np.array([4, 5, 6], np.int32))
        assert np.array_equal(good.result(timeout=5), _logits(np.array([4, 5, 6], np.int32)))


def test_masks_pass_through_and_close():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel()
    s = StreamingScheduler([m], max_tokens=50, max_wait_ms=50)
    ids = np.array([4, 5, 6, 1], np.int32)
    mask = np.array([1, 1, 1, 0], np.int32)
    f1 = s.submit(ids, mask)
    f2 = s.submit(ids)
    s.close()  # flushes what was submitted
    assert np.array_equal(f1.result(timeout=1), _logits(ids, mask))
    assert np.array_equal(f2.result(timeout=1), _logits(ids, np.ones_like(ids)))
    with pytest.raises(RuntimeError, match="closed"):
        s.submit(ids)
    with pytest.raises(ValueError):
        StreamingScheduler([])


def test_cancelled_requests_are_skipped():
    from esm_b200.streaming import StreamingScheduler

    m = FakeModel()
    s = StreamingScheduler([m], max_tokens=10**6, max_wait_ms=200)
    keep = s.submit(np.array([4, 5], np.int32))
    drop = s.submit(np.array([6, 7, 8], np.int32))
    assert drop.cancel()
    s.close()
    assert np.array_equal(keep.result(timeout=1), _logits(np.array([4, 5], np.int32)))
    assert drop.cancelled()
    assert m.batches == [[2]]
