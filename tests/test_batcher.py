"""The dynamic batcher (host side, no GPU): flush on size, on timeout and on a token
budget; results in order; failures fanned out to every caller of the batch; queued
requests failed on stop (the reference's DynamicBatcher, deploy/server/batcher.py:39)."""

from __future__ import annotations

import asyncio
import threading
import time

import pytest

from latefuse_b200.batcher import DynamicBatcher, InferenceResult, token_cost


def echo_fn(log):
    def fn(batch):
        log.append([r.text for r in batch])
        return [InferenceResult(scores=[float(len(r.text))], latency_ms=0.0) for r in batch]
    return fn


def run(coro):
    return asyncio.run(coro)


def test_full_batches_flush_without_waiting_for_the_timeout():
    log = []

    async def main():
        b = DynamicBatcher(max_batch_size=4, batch_timeout_ms=10_000, inference_fn=echo_fn(log))
        await b.start()
        t0 = time.monotonic()
        res = await asyncio.gather(*(b.submit(f"t{i}", "x" * i) for i in range(8)))
        took = time.monotonic() - t0
        await b.stop()
        return res, took

    res, took = run(main())
    assert [r.scores[0] for r in res] == [float(i) for i in range(8)]  # each caller gets its own row
    assert sorted(len(x) for x in log) == [4, 4]
    assert took < 5.0


def test_partial_batch_flushes_on_timeout():
    log = []

    async def main():
        b = DynamicBatcher(max_batch_size=64, batch_timeout_ms=20, inference_fn=echo_fn(log))
        await b.start()
        res = await asyncio.gather(b.submit("a", "one"), b.submit("b", "three"))
        await b.stop()
        return res

    res = run(main())
    assert [r.scores for r in res] == [[3.0], [5.0]]
    assert log == [["one", "three"]]


def test_token_budget_closes_a_batch_and_the_overflowing_request_opens_the_next():
    log = []

    async def main():
        b = DynamicBatcher(max_batch_size=64, batch_timeout_ms=50, inference_fn=echo_fn(log),
                           max_batch_tokens=10, cost_fn=token_cost)
        await b.start()
        reqs = [b.submit("t", f"r{i}", payload=n) for i, n in enumerate([4, 4, 4, 9, 1])]
        res = await asyncio.gather(*reqs)
        await b.stop()
        return res

    res = run(main())
    assert len(res) == 5
    assert log == [["r0", "r1"], ["r2"], ["r3", "r4"]]  # 4+4 | 4 (+9 > 10) | 9+1


def test_a_failing_forward_fails_every_caller_of_its_batch_only():
    calls = []

    def fn(batch):
        calls.append(len(batch))
        if any(r.text == "boom" for r in batch):
            raise ValueError("bad batch")
        return [InferenceResult(scores=[1.0], latency_ms=0.0) for _ in batch]

    async def main():
        b = DynamicBatcher(max_batch_size=2, batch_timeout_ms=1000, inference_fn=fn)
        await b.start()
        first = await asyncio.gather(b.submit("t", "boom"), b.submit("t", "ok"), return_exceptions=True)
        second = await asyncio.gather(b.submit("t", "fine"), b.submit("t", "fine"))
        await b.stop()
        return first, second

    first, second = run(main())
    assert all(isinstance(e, ValueError) for e in first)
    assert [r.scores for r in second] == [[1.0], [1.0]]


def test_wrong_result_count_is_an_error_for_the_batch():
    async def main():
        b = DynamicBatcher(max_batch_size=2, batch_timeout_ms=1000,
                           inference_fn=lambda batch: [InferenceResult([0.0], 0.0)])
        await b.start()
        out = await asyncio.gather(b.submit("t", "a"), b.submit("t", "b"), return_exceptions=True)
        await b.stop()
        return out

    out = run(main())
    assert all(isinstance(e, RuntimeError) and "returned 1 results" in str(e) for e in out)


def test_coroutine_inference_fn_and_stop_fails_queued_requests():
    gate = asyncio.Event

    async def main():
        release = gate()

        async def fn(batch):
            await release.wait()
            return [InferenceResult([1.0], 0.0) for _ in batch]

        b = DynamicBatcher(max_batch_size=1, batch_timeout_ms=0, inference_fn=fn)
        await b.start()
        t1 = asyncio.ensure_future(b.submit("t", "a"))   # runs, blocked on the gate
        t2 = asyncio.ensure_future(b.submit("t", "b"))   # stays queued
        await asyncio.sleep(0.05)
        await b.stop()
        release.set()
        return await asyncio.gather(t1, t2, return_exceptions=True)

    out = run(main())
    assert isinstance(out[0], RuntimeError) and "while this request ran" in str(out[0])
    assert isinstance(out[1], RuntimeError) and "before this request ran" in str(out[1])


def test_cancelled_requests_are_dropped_before_the_forward():
    log = []

    async def main():
        b = DynamicBatcher(max_batch_size=8, batch_timeout_ms=100, inference_fn=echo_fn(log))
        await b.start()
        gone = asyncio.ensure_future(b.submit("t", "gone"))
        kept = asyncio.ensure_future(b.submit("t", "kept"))
        await asyncio.sleep(0.01)
        gone.cancel()
        res = await kept
        await b.stop()
        return res

    assert run(main()).scores == [4.0]
    assert log == [["kept"]]


def test_classifier_inference_fn_returns_each_rows_logits_under_the_lock():
    class FakeClassifier:
        def __init__(self):
            self.calls = []

        def logits(self, texts, tenants):
            self.calls.append((list(texts), list(tenants)))
            return [[float(len(t)), float(i)] for i, t in enumerate(texts)]

    from latefuse_b200.batcher import classifier_inference_fn

    clf, lock = FakeClassifier(), threading.Lock()

    async def main():
        b = DynamicBatcher(4, 20, classifier_inference_fn(clf, lock))
        await b.start()
        out = await asyncio.gather(b.submit("a", "xx"), b.submit("b", "yyy"))
        await b.stop()
        return out

    out = run(main())
    assert [r.scores for r in out] == [[2.0, 0.0], [3.0, 1.0]]
    assert clf.calls == [(["xx", "yyy"], ["a", "b"])]
    assert not lock.locked()


def test_submit_before_start_and_bad_arguments_raise():
    with pytest.raises(ValueError):
        DynamicBatcher(0, 1.0, lambda b: [])
    with pytest.raises(ValueError):
        DynamicBatcher(4, -1.0, lambda b: [])

    async def main():
        b = DynamicBatcher(4, 1.0, lambda b: [])
        with pytest.raises(RuntimeError, match="start"):
            await b.submit("t", "x")

    run(main())


def test_forward_runs_off_the_event_loop_thread():
    seen = []

    def fn(batch):
        seen.append(threading.current_thread() is threading.main_thread())
        return [InferenceResult([0.0], 0.0) for _ in batch]

    async def main():
        b = DynamicBatcher(8, 1.0, fn)
        await b.start()
        await b.submit("t", "x")
        await b.stop()

    run(main())
    assert seen == [False]
