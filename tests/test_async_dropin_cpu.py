"""The reference's AsyncInferenceEngine runs unchanged on this package's scheduler.

The reference's asyncio front (generation/async_engine.py:77-239) builds its
scheduler from the name ``ContinuousBatchingScheduler`` imported into its
module.  Binding that name to this package's scheduler -- the one-line import
change a maintainer would make -- is done here with ``monkeypatch``; the
reference engine's code is otherwise untouched.  Scenarios follow the
reference's own tests/test_async_inference_engine.py:16-160 (streaming with
EOS, prefill failure routed to its handle, wake after idle, cancel and
idempotent close), with a scripted model that only does cache accounting, so
the scheduler runs on host caches without kernels.

The reference is imported from the checkout named by NIE_REFERENCE_SRC (its
``src`` directory); without it the tests skip.
"""

import asyncio
import os
import sys

import pytest
import torch

from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
from nano_infer_engine_b200.paged_cache import PagedKVCache

REF = os.environ.get("NIE_REFERENCE_SRC")
pytestmark = pytest.mark.skipif(not REF, reason="NIE_REFERENCE_SRC (reference checkout's src) not set")
EOS = 2


@pytest.fixture()
def ref_async(monkeypatch):
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from nano_infer_engine.generation import async_engine

    monkeypatch.setattr(async_engine, "ContinuousBatchingScheduler", ContinuousBatchingScheduler)
    return async_engine


class _Scripted:
    """One-hot logits from a per-request token schedule; cache accounting only."""

    def __init__(self, schedules, failing_prefill=None):
        self.schedules = schedules
        self.at = {s: 0 for s in schedules}
        self.failing_prefill = failing_prefill

    def __call__(self, input_ids, *, kv_cache, sequence_id="default", sequence_ids=None):
        ids = sequence_ids or (sequence_id,)
        logits = torch.zeros(len(ids), input_ids.shape[1], 8)
        for row, sid in enumerate(ids):
            have = kv_cache.get_sequence_length(sid)
            steps = input_ids.shape[1] if have == 0 else 1
            kv_cache.ensure_capacity(sid, have + steps)
            kv_cache.advance(sid, steps)
            if sid == self.failing_prefill and have == 0:
                raise RuntimeError("prefill failed")
            logits[row, -1, self.schedules[sid][self.at[sid]]] = 1.0
            self.at[sid] += 1
        return logits


def _engine(async_engine, model, max_new_tokens, eos=EOS):
    from nano_infer_engine_b200.generation.config import GenerationConfig

    cache = PagedKVCache(max_new_tokens * 2, 1, 1, 1, 1, torch.float32, "cpu")
    config = GenerationConfig(max_new_tokens=max_new_tokens, eos_token_id=eos, use_cache=True)
    engine = async_engine.AsyncInferenceEngine(model, config, cache, max_batch_size=2)
    assert isinstance(engine.scheduler, ContinuousBatchingScheduler)
    return engine, cache


async def _collect(handle):
    return [event async for event in handle], await handle.result()


def _generated(result):
    return tuple(result.sequence[0, 1:].tolist())  # every prompt here is one token


def test_reference_async_engine_streams_our_scheduler_tokens(ref_async):
    from nano_infer_engine_b200.generation.events import TokenEvent
    from nano_infer_engine_b200.generation.request import RequestStatus

    async def scenario():
        engine, cache = _engine(ref_async, _Scripted({"request-a": (3, EOS), "request-b": (4, 5, EOS)}), 3)
        a = await engine.submit(torch.tensor([[1]]), sequence_id="request-a")
        b = await engine.submit(torch.tensor([[1]]), sequence_id="request-b")
        (ev_a, res_a), (ev_b, res_b) = await asyncio.gather(_collect(a), _collect(b))
        assert ev_a == [TokenEvent("request-a", 3), TokenEvent("request-a", EOS)]
        assert ev_b == [TokenEvent("request-b", 4), TokenEvent("request-b", 5), TokenEvent("request-b", EOS)]
        assert res_a.status is RequestStatus.COMPLETED and res_b.status is RequestStatus.COMPLETED
        assert _generated(res_b) == (4, 5, EOS) and res_b.stopped_by_eos
        assert cache.allocator.allocated_block_count == 0
        await engine.close()

    asyncio.run(scenario())


def test_reference_async_engine_routes_prefill_failure_to_its_handle(ref_async):
    from nano_infer_engine_b200.generation.request import RequestStatus

    async def scenario():
        model = _Scripted({"request-a": (3,), "request-b": (4, 5)}, failing_prefill="request-a")
        engine, cache = _engine(ref_async, model, 2, eos=None)
        bad = await engine.submit(torch.tensor([[1]]), sequence_id="request-a")
        good = await engine.submit(torch.tensor([[1]]), sequence_id="request-b")
        (ev_bad, res_bad), (ev_good, res_good) = await asyncio.gather(_collect(bad), _collect(good))
        assert ev_bad == [] and res_bad.status is RequestStatus.FAILED
        assert isinstance(res_bad.error, RuntimeError)
        assert res_good.status is RequestStatus.COMPLETED and _generated(res_good) == (4, 5)
        assert cache.allocator.allocated_block_count == 0
        await engine.close()

    asyncio.run(scenario())


def test_reference_async_engine_wakes_after_idle_cancels_and_closes(ref_async):
    from nano_infer_engine_b200.generation.request import RequestStatus

    async def scenario():
        model = _Scripted({"request-a": (3, 4), "request-b": (5, 6), "request-c": (7, 7, 7, 7, 7, 7)})
        engine, cache = _engine(ref_async, model, 2, eos=None)
        first = await engine.submit(torch.tensor([[1]]), sequence_id="request-a")
        assert _generated(await first.result()) == (3, 4)
        await asyncio.sleep(0.05)  # the worker goes idle, then must wake for new work
        second = await engine.submit(torch.tensor([[1]]), sequence_id="request-b")
        assert _generated(await second.result()) == (5, 6)
        assert cache.allocator.allocated_block_count == 0
        await engine.close()
        assert engine.is_closed
        await engine.close()  # idempotent

        engine, cache = _engine(ref_async, model, 6, eos=None)
        third = await engine.submit(torch.tensor([[1]]), sequence_id="request-c")
        assert await third.cancel() in (True, False)  # cancelled, unless it already finished
        result = await third.result()
        assert result.status in (RequestStatus.CANCELLED, RequestStatus.COMPLETED)
        await engine.close()
        assert cache.allocator.allocated_block_count == 0

    asyncio.run(scenario())
