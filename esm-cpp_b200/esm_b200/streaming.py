"""Streaming submit/future front end over Model.forward_scheduled.

The reference exposes only the synchronous Model::ForwardScheduled (model.h:
152-159) and lists a streaming submit/future API as its next version
(docs/architecture.md:76).  This is that front end for one or more models (one
per GPU), packing requests from any number of callers:

  - submit() queues one sequence and returns a concurrent.futures.Future whose
    result is that sequence's logits [L, V];
  - a dispatcher thread cuts the pending queue into batches of at most
    `max_tokens` tokens, as soon as that many are pending or the oldest
    request has waited `max_wait_ms`;
  - each batch goes to the least-loaded model's worker thread, which runs
    forward_scheduled on it (PlanBatches grouping inside); the forward
    releases the GIL, so one thread per GPU keeps every device busy.

Numerics: a request's logits are those of forward_scheduled on the batch it
was packed into.  With the per-tensor W8A8 activation scale the group
membership is part of the result, as it is for ForwardScheduled itself;
per-token activation quantisation (Model.set_act_quant("per_token")) and FP32
models make each sequence's logits independent of its batch mates up to FP32
rounding.
"""
from __future__ import annotations

import threading
import time
from collections import deque
from concurrent.futures import Future

import numpy as np


class StreamingScheduler:
    """Cross-request packing over `models` (objects with Model's
    forward_scheduled signature)."""

    def __init__(self, models, max_tokens: int = 32768, max_wait_ms: float = 5.0,
                 imbalance_threshold: float = 1.2, max_batch_size: int = 256):
        models = list(models)
        if not models:
            raise ValueError("StreamingScheduler needs at least one model")
        if max_tokens <= 0:
            raise ValueError("max_tokens must be positive")
        self._models = models
        self._max_tokens = int(max_tokens)
        self._max_wait = float(max_wait_ms) / 1000.0
        self._threshold = float(imbalance_threshold)
        self._max_batch = int(max_batch_size)
        self._cv = threading.Condition()
        self._pending: deque = deque()  # (ids, mask, future, t_submit)
        self._pending_tokens = 0
        self._closed = False
        self._load = [0] * len(models)  # tokens queued or running per model
        self._queues = [deque() for _ in models]
        self._workers = [threading.Thread(target=self._work, args=(i,), daemon=True,
                                          name=f"esm-stream-{i}") for i in range(len(models))]
        self._dispatcher = threading.Thread(target=self._dispatch, daemon=True,
                                            name="esm-stream-dispatch")
        for t in self._workers:
            t.start()
        self._dispatcher.start()

    # ----------------------------------------------------------- callers
    def submit(self, input_ids, attention_mask=None) -> Future:
        """Queues one sequence; the future's result is its logits [L, V]."""
        ids = np.ascontiguousarray(input_ids, np.int32)
        if ids.ndim != 1:
            raise ValueError("input_ids must be a 1-D int32 array")
        mask = None
        if attention_mask is not None:
            mask = np.ascontiguousarray(attention_mask, np.int32)
            if mask.shape != ids.shape:
                raise ValueError("attention_mask must have the shape of input_ids")
        fut: Future = Future()
        with self._cv:
            if self._closed:
                raise RuntimeError("StreamingScheduler is closed")
            self._pending.append((ids, mask, fut, time.monotonic()))
            self._pending_tokens += ids.shape[0]
            self._cv.notify_all()
        return fut

    def submit_many(self, input_ids, attention_masks=None) -> list:
        masks = attention_masks if attention_masks is not None else [None] * len(input_ids)
        return [self.submit(ids, m) for ids, m in zip(input_ids, masks)]

    def close(self, wait: bool = True) -> None:
        """Stops accepting requests; everything already submitted still runs."""
        with self._cv:
            self._closed = True
            self._cv.notify_all()
        if wait:
            self._dispatcher.join()
            for t in self._workers:
                t.join()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---------------------------------------------------------- internals
    def _take_batch(self):
        """Pops up to max_tokens tokens of pending requests (at least one)."""
        batch, tokens = [], 0
        while self._pending:
            n = self._pending[0][0].shape[0]
            if batch and tokens + n > self._max_tokens:
                break
            batch.append(self._pending.popleft())
            tokens += n
        self._pending_tokens -= tokens
        return batch, tokens

    def _dispatch(self):
        while True:
            with self._cv:
                while True:
                    if self._pending:
                        age = time.monotonic() - self._pending[0][3]
                        if (self._pending_tokens >= self._max_tokens or age >= self._max_wait
                                or self._closed):
                            break
                        self._cv.wait(timeout=self._max_wait - age)
                    elif self._closed:
                        for q in self._queues:
                            q.append(None)  # workers drain their queue, then stop
                        self._cv.notify_all()
                        return
                    else:
                        self._cv.wait()
                batch, tokens = self._take_batch()
                w = min(range(len(self._models)), key=lambda i: self._load[i])
                self._load[w] += tokens
                self._queues[w].append((batch, tokens))
                self._cv.notify_all()

    def _work(self, i: int):
        model = self._models[i]
        while True:
            with self._cv:
                while not self._queues[i]:
                    self._cv.wait()
                item = self._queues[i].popleft()
            if item is None:
                return
            batch, tokens = item
            live = [r for r in batch if r[2].set_running_or_notify_cancel()]
            try:
                if live:
                    masks = None
                    if any(r[1] is not None for r in live):
                        masks = [r[1] if r[1] is not None else np.ones_like(r[0]) for r in live]
                    out = model.forward_scheduled([r[0] for r in live], masks,
                                                  imbalance_threshold=self._threshold,
                                                  max_batch_size=self._max_batch)
                    for r, lg in zip(live, out):
                        r[2].set_result(lg)
            except BaseException as e:  # noqa: BLE001 -- delivered to the callers
                for r in live:
                    if not r[2].done():
                        r[2].set_exception(e)
            finally:
                with self._cv:
                    self._load[i] -= tokens
