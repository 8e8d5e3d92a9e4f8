"""Asynchronous dynamic batcher: single requests in, one forward per batch out.

The serving front end of the reference (``deploy/server/batcher.py:39``,
``DynamicBatcher`` with ``start`` / ``stop`` / ``submit``, and its inference
function ``deploy/server/app.py:70-94``) collects single HTTP requests until a
batch is full or a timeout passes, runs the model once on the batch in a worker
thread, and resolves each caller's future with its row.  This module keeps that
interface (the same class, method and record names, the same flush rule and error
fan-out) for the padding-free forward this library runs:

* a batch is also closed by a **token budget** (``max_batch_tokens``, counted by
  ``cost_fn``): the packed forward's cost follows real tokens, not rows, so a
  budget keeps the step time even when request lengths vary;
* requests that arrive while a batch runs are collected immediately after it (the
  queue is drained without waiting before the timeout clock starts);
* ``stop`` fails the requests still queued with ``RuntimeError`` instead of
  leaving their callers waiting forever;
* a request whose caller stopped waiting (a cancelled future) is dropped from the
  batch before the forward.

The model call itself stays synchronous (GPU-bound) and runs in the loop's default
executor, as the reference's does, so the event loop keeps accepting requests.
"""

from __future__ import annotations

import asyncio
import logging
import inspect
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Sequence

logger = logging.getLogger(__name__)


@dataclass
class InferenceRequest:
    """One caller's input, waiting for a batch.  ``payload`` carries anything extra
    the inference function needs (pre-tokenized ids, a text pair, ...)."""

    tenant_id: str
    text: str
    payload: Any = None
    future: asyncio.Future | None = None
    enqueued_at: float = field(default_factory=time.monotonic)


@dataclass
class InferenceResult:
    """One row of a batch's output and the batch's forward latency."""

    scores: list[float]
    latency_ms: float


InferenceFn = Callable[[list[InferenceRequest]], Sequence[InferenceResult]]


def _default_cost(req: InferenceRequest) -> int:
    return 1


class DynamicBatcher:
    """Collect requests into batches and run ``inference_fn`` once per batch.

    A batch closes when it holds ``max_batch_size`` requests, when adding the next
    request would pass ``max_batch_tokens`` (if set; measured by ``cost_fn``, e.g.
    the request's token count), or ``batch_timeout_ms`` after its first request
    arrived.  ``inference_fn`` takes the list of requests and returns one
    :class:`InferenceResult` per request, in order; it may be a plain function (run
    in the event loop's executor) or a coroutine function.  If it raises, or returns
    the wrong number of results, every request of the batch gets the exception.

        batcher = DynamicBatcher(max_batch_size=64, batch_timeout_ms=5.0, inference_fn=fn)
        await batcher.start()
        result = await batcher.submit("tenant_42", "some text")
        await batcher.stop()
    """

    def __init__(self, max_batch_size: int, batch_timeout_ms: float, inference_fn: InferenceFn, *,
                 max_batch_tokens: int | None = None,
                 cost_fn: Callable[[InferenceRequest], int] = _default_cost):
        if max_batch_size < 1:
            raise ValueError(f"max_batch_size must be at least 1, got {max_batch_size}")
        if batch_timeout_ms < 0:
            raise ValueError(f"batch_timeout_ms must be non-negative, got {batch_timeout_ms}")
        if max_batch_tokens is not None and max_batch_tokens < 1:
            raise ValueError(f"max_batch_tokens must be at least 1, got {max_batch_tokens}")
        self._max_batch_size = max_batch_size
        self._batch_timeout_ms = batch_timeout_ms
        self._inference_fn = inference_fn
        self._max_tokens = max_batch_tokens
        self._cost = cost_fn
        self._queue: asyncio.Queue[InferenceRequest] | None = None
        self._held: InferenceRequest | None = None  # closed the last batch by its token cost
        self._task: asyncio.Task | None = None
        self._running = False
        #: batches run and requests served so far
        self.batches = 0
        self.served = 0

    @property
    def running(self) -> bool:
        return self._running

    async def start(self) -> None:
        """Start the batching loop on the running event loop."""
        if self._running:
            return
        self._queue = asyncio.Queue()
        self._running = True
        self._task = asyncio.get_running_loop().create_task(self._loop())
        logger.info("batcher started (max_batch=%d, timeout=%.1f ms, max_tokens=%s)", self._max_batch_size,
                    self._batch_timeout_ms, self._max_tokens)

    async def stop(self) -> None:
        """Stop the loop; requests still queued fail with ``RuntimeError``."""
        self._running = False
        if self._task is not None:
            self._task.cancel()
            try:
                await self._task
            except asyncio.CancelledError:
                pass
            self._task = None
        pending = [self._held] if self._held is not None else []
        self._held = None
        while self._queue is not None and not self._queue.empty():
            pending.append(self._queue.get_nowait())
        for req in pending:
            if req.future is not None and not req.future.done():
                req.future.set_exception(RuntimeError("the batcher was stopped before this request ran"))
        logger.info("batcher stopped (%d batches, %d requests)", self.batches, self.served)

    async def submit(self, tenant_id: str, text: str, payload: Any = None) -> InferenceResult:
        """Queue one request and wait for its row of the batch it lands in."""
        if not self._running or self._queue is None:
            raise RuntimeError("the batcher is not running: await start() first")
        req = InferenceRequest(tenant_id=tenant_id, text=text, payload=payload,
                               future=asyncio.get_running_loop().create_future())
        await self._queue.put(req)
        return await req.future

    # -- the loop ------------------------------------------------------------
    async def _next_batch(self) -> list[InferenceRequest]:
        """Wait for a first request, then gather until full, over budget or timed out."""
        assert self._queue is not None
        first = self._held if self._held is not None else await self._queue.get()
        self._held = None
        batch, tokens = [first], self._cost(first)
        deadline = time.monotonic() + self._batch_timeout_ms / 1000.0

        def take(req: InferenceRequest) -> bool:
            nonlocal tokens
            cost = self._cost(req)
            if self._max_tokens is not None and tokens + cost > self._max_tokens:
                self._held = req  # it opens the next batch
                return False
            batch.append(req)
            tokens += cost
            return True

        while len(batch) < self._max_batch_size:
            if not self._queue.empty():  # already waiting: no need to wait for it
                if not take(self._queue.get_nowait()):
                    break
                continue
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                break
            try:
                req = await asyncio.wait_for(self._queue.get(), timeout=remaining)
            except asyncio.TimeoutError:
                break
            if not take(req):
                break
        return batch

    async def _loop(self) -> None:
        while self._running:
            batch = await self._next_batch()
            live = [r for r in batch if r.future is None or not r.future.done()]
            if live:
                await self._run(live)

    async def _run(self, batch: list[InferenceRequest]) -> None:
        t0 = time.monotonic()
        try:
            results = await self._forward(batch)
        except asyncio.CancelledError:  # stopped mid-batch: its callers must not wait forever
            for req in batch:
                if req.future is not None and not req.future.done():
                    req.future.set_exception(RuntimeError("the batcher was stopped while this request ran"))
            raise
        if results is None:
            return
        self.batches += 1
        self.served += len(batch)
        logger.debug("batch of %d in %.1f ms", len(batch), (time.monotonic() - t0) * 1e3)
        for req, res in zip(batch, results):
            if req.future is not None and not req.future.done():
                req.future.set_result(res)

    async def _forward(self, batch: list[InferenceRequest]) -> list[InferenceResult] | None:
        """The batch's results, or None after failing every request with the error."""
        try:
            if inspect.iscoroutinefunction(self._inference_fn):
                results = await self._inference_fn(batch)
            else:
                results = await asyncio.get_running_loop().run_in_executor(None, self._inference_fn, batch)
            results = list(results)
            if len(results) != len(batch):
                raise RuntimeError(f"inference_fn returned {len(results)} results for a batch of {len(batch)}")
        except Exception as exc:  # every caller of the batch sees the failure
            logger.error("batch of %d failed: %s", len(batch), exc)
            for req in batch:
                if req.future is not None and not req.future.done():
                    req.future.set_exception(exc)
            return None
        return results


def classifier_inference_fn(classifier, lock=None) -> InferenceFn:
    """An ``inference_fn`` serving a :class:`~latefuse_b200.tasks.MultiTenantClassifier`:
    each request's text under its tenant's adapter and head, the row's logits as
    scores (the reference server's ``run_inference``, ``deploy/server/app.py:70-94``).
    ``lock`` (a ``threading.Lock``) serialises the forward against adapter reloads."""
    import contextlib

    def run(batch: list[InferenceRequest]) -> list[InferenceResult]:
        t0 = time.monotonic()
        with lock if lock is not None else contextlib.nullcontext():
            scores = classifier.logits([r.text for r in batch], [r.tenant_id for r in batch])
        ms = (time.monotonic() - t0) * 1e3
        return [InferenceResult(scores=list(row), latency_ms=ms) for row in scores]

    return run


def token_cost(req: InferenceRequest) -> int:
    """``cost_fn`` for requests whose ``payload`` is their token ids (or a length)."""
    p = req.payload
    if p is None:
        return max(1, len(req.text.split()))
    return int(p) if isinstance(p, int) else len(p)


__all__ = ["DynamicBatcher", "InferenceRequest", "InferenceResult", "classifier_inference_fn", "token_cost"]
