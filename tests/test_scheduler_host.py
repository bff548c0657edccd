"""Scheduler step plans on the host (CPU caches, scripted models, no kernels).

The expected values are the reference's own assertions for the same
scenarios (nano_infer_engine tests/test_paged_greedy_generation.py:530-729):
ragged order = prefill chunks first, then decode tokens; the round-robin
prefill budget; one chunk per step; admission and failure isolation.
"""

import pytest
import torch

from nano_infer_engine_b200.generation.config import GenerationConfig
from nano_infer_engine_b200.generation.paged_prefill import paged_prefill, paged_prefill_chunks
from nano_infer_engine_b200.generation.request import PagedRequest, RequestStatus
from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
from nano_infer_engine_b200.paged_cache import PagedKVCache

VOCAB = 8


class ScriptedModel:
    """Cache accounting plus one-hot logits; records every ragged call."""

    def __init__(self, schedules=None, max_seq_len=64):
        self.schedules = schedules or {}
        self.next_index: dict[str, int] = {}
        self.ragged_calls: list[tuple[tuple[str, ...], tuple[int, ...]]] = []
        self.decode_calls: list[tuple[str, ...]] = []

        class _Cfg:
            pass

        self.config = _Cfg()
        self.config.max_seq_len = max_seq_len

    def _token(self, sid):
        sched = self.schedules.get(sid, (1,))
        i = self.next_index.get(sid, 0)
        self.next_index[sid] = i + 1
        return sched[min(i, len(sched) - 1)]

    def forward_ragged(self, input_ids, *, kv_cache, sequence_ids, query_start_loc):
        bounds = query_start_loc.tolist()
        self.ragged_calls.append((tuple(sequence_ids), tuple(bounds)))
        logits = torch.zeros(input_ids.numel(), VOCAB)
        for sid, a, b in zip(sequence_ids, bounds, bounds[1:]):
            n = kv_cache.get_sequence_length(sid)
            kv_cache.ensure_capacity(sid, n + b - a)
            kv_cache.advance(sid, b - a)
            logits[b - 1, self._token(sid)] = 1.0
        return logits

    def __call__(self, input_ids, *, kv_cache, sequence_id="default", sequence_ids=None):
        ids = sequence_ids or (sequence_id,)
        steps = input_ids.shape[1]
        if steps == 1 and all(kv_cache.get_sequence_length(s) > 0 for s in ids):
            self.decode_calls.append(tuple(ids))
        logits = torch.zeros(len(ids), steps, VOCAB)
        for i, sid in enumerate(ids):
            n = kv_cache.get_sequence_length(sid)
            kv_cache.ensure_capacity(sid, n + steps)
            kv_cache.advance(sid, steps)
            logits[i, -1, self._token(sid)] = 1.0
        return logits


def _cache(num_blocks, block_size=1):
    return PagedKVCache(num_blocks, block_size, 1, 1, 4, torch.float32, "cpu")


def test_request_initial_state():
    prompt = torch.tensor([[1, 4]])
    r = PagedRequest(sequence_id="request-a", prompt=prompt)
    assert r.sequence is prompt
    assert (r.generated_tokens, r.finished, r.status, r.error) == (0, False, RequestStatus.PENDING, None)
    r.append_token(5)
    assert r.sequence.tolist() == [[1, 4, 5]]


def test_unified_step_orders_prefill_before_decode():
    model = ScriptedModel()
    cache = _cache(12)
    s = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=2, prefill_chunk_size=2), cache, 2)
    a = s.add_request("request-a", torch.tensor([[1]]))
    b = s.add_request("request-b", torch.tensor([[2, 3, 4, 5]]))
    s.step()
    assert a.status is RequestStatus.ACTIVE and b.status is RequestStatus.PREFILLING
    model.ragged_calls.clear()
    out = s.step()
    assert model.ragged_calls == [(("request-b", "request-a"), (0, 2, 3))]
    assert out.token_events[0].sequence_id == "request-a"
    assert b.status is RequestStatus.ACTIVE


def test_round_robin_prefill_budget():
    model = ScriptedModel()
    cache = _cache(24)
    s = ContinuousBatchingScheduler(
        model, GenerationConfig(max_new_tokens=1, prefill_chunk_size=2, max_prefill_tokens_per_step=3), cache, 3
    )
    reqs = [s.add_request(f"request-{i}", torch.tensor([[1, 2, 3, 4, 5, 6]])) for i in range(3)]
    s.step()
    assert tuple(r.prefill_offset for r in reqs) == (2, 1, 0)
    s.step()
    assert tuple(r.prefill_offset for r in reqs) == (3, 1, 2)
    s.step()
    assert tuple(r.prefill_offset for r in reqs) == (3, 3, 3)


def test_chunked_prefill_advances_once_per_step():
    model = ScriptedModel()
    cache = _cache(8)
    s = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=1, prefill_chunk_size=2), cache, 1)
    r = s.add_request("request-a", torch.tensor([[1, 2, 3, 4, 5]]))
    nxt = s.add_request("request-b", torch.tensor([[6]]))
    assert s.step().token_events == ()
    assert (r.status, r.prefill_offset, cache.get_sequence_length("request-a")) == (RequestStatus.PREFILLING, 2, 2)
    assert s.step().token_events == ()
    assert r.prefill_offset == 4
    out = s.step()
    assert out.token_events == () and r.status is RequestStatus.ACTIVE and r.prefill_offset == 5
    out = s.step()
    assert len(out.token_events) == 1 and out.terminal_requests == (r,)
    assert nxt.status is RequestStatus.PENDING and s.pending_count == 1
    assert s.step().token_events == () and nxt.status is RequestStatus.ACTIVE
    assert s.step().terminal_requests == (nxt,)
    assert not s.has_work and cache.allocator.allocated_block_count == 0


def test_eos_and_token_limit_release_blocks():
    model = ScriptedModel({"a": (3, 7, 7), "b": (2, 2, 2, 2)})
    cache = _cache(32, block_size=2)
    s = ContinuousBatchingScheduler(
        model, GenerationConfig(max_new_tokens=3, eos_token_id=7, prefill_chunk_size=4), cache, 2
    )
    a = s.add_request("a", torch.tensor([[1, 2, 3]]))
    b = s.add_request("b", torch.tensor([[4, 5]]))
    s.run_until_idle()
    assert a.sequence[0, 3:].tolist() == [3, 7] and a.finished
    assert b.sequence[0, 2:].tolist() == [2, 2, 2] and not b.finished
    assert cache.allocator.allocated_block_count == 0
    assert s.reserved_blocks == 0


def test_non_chunked_mode_batches_decode():
    model = ScriptedModel({"a": (1, 2, 3), "b": (4, 5, 6)})
    cache = _cache(32, block_size=2)
    s = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=3), cache, 2)
    a = s.add_request("a", torch.tensor([[1, 2]]))
    b = s.add_request("b", torch.tensor([[3, 4, 5]]))
    s.run_until_idle()
    assert a.sequence[0, 2:].tolist() == [1, 2, 3]
    assert b.sequence[0, 3:].tolist() == [4, 5, 6]
    assert model.decode_calls[0] == ("a", "b")


def test_failed_ragged_step_fails_its_requests():
    class Failing(ScriptedModel):
        def forward_ragged(self, *args, **kwargs):
            raise RuntimeError("boom")

    cache = _cache(16)
    s = ContinuousBatchingScheduler(Failing(), GenerationConfig(max_new_tokens=2, prefill_chunk_size=2), cache, 2)
    r = s.add_request("a", torch.tensor([[1, 2, 3]]))
    out = s.step()
    assert out.terminal_requests == (r,) and r.status is RequestStatus.FAILED
    assert isinstance(r.error, RuntimeError) and s.reserved_blocks == 0


def test_admission_validations():
    model = ScriptedModel(max_seq_len=8)
    cache = _cache(4)
    s = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=4, prefill_chunk_size=2), cache, 1)
    with pytest.raises(ValueError, match="exceeds max model length"):
        s.add_request("a", torch.tensor([[1] * 6]))
    with pytest.raises(ValueError, match="cannot fit in paged cache"):
        ContinuousBatchingScheduler(ScriptedModel(), GenerationConfig(max_new_tokens=4), _cache(4), 1).add_request(
            "b", torch.tensor([[1, 2]])
        )
    s.add_request("c", torch.tensor([[1]]))
    with pytest.raises(ValueError, match="already submitted"):
        s.add_request("c", torch.tensor([[1]]))
    assert s.cancel_request("c") and s.get_request("c").status is RequestStatus.CANCELLED
    s.close()
    with pytest.raises(RuntimeError, match="scheduler is closed"):
        s.step()


def test_prefill_chunks_contract_with_foreign_models():
    """A model that ignores the last-row request still gets indexed like the reference."""
    model = ScriptedModel({"x": (5,), "y": (6,)})
    cache = _cache(16)
    logits = paged_prefill_chunks(model, (torch.tensor([[1, 2, 3]]), torch.tensor([[4]])), cache, ("x", "y"))
    assert logits.shape == (2, VOCAB) and logits.argmax(-1).tolist() == [5, 6]
    assert model.ragged_calls == [(("x", "y"), (0, 3, 4))]
    out = paged_prefill(ScriptedModel({"p": (2,), "q": (3,)}), (torch.tensor([[1, 2]]), torch.tensor([[1]])),
                        _cache(8), ("p", "q"))
    assert out.argmax(-1).tolist() == [2, 3]
    with pytest.raises(ValueError, match="must have the same length"):
        paged_prefill(model, (torch.tensor([[1]]),), _cache(4), ("a", "b"))
    with pytest.raises(ValueError, match="sequence IDs must be unique"):
        paged_prefill(model, (torch.tensor([[1]]), torch.tensor([[2]])), _cache(4), ("a", "a"))


def test_retire_by_count_defers_the_token_appends():
    """Without token values (no EOS configured) retirement goes by count and the caller appends later."""
    cache = _cache(32, block_size=2)
    s = ContinuousBatchingScheduler(ScriptedModel(), GenerationConfig(max_new_tokens=2), cache, 2)
    reqs = [PagedRequest(sequence_id=sid, prompt=torch.tensor([[1, 2]])) for sid in ("a", "b")]
    reqs[1].generated_tokens = 1
    done: list = []
    keep = s._retire(reqs, None, done)
    assert keep == [0] and done == [reqs[1]]
    assert [r.generated_tokens for r in reqs] == [1, 2]
    assert all(r.sequence.shape[1] == 2 for r in reqs)  # nothing appended yet
    s_eos = ContinuousBatchingScheduler(ScriptedModel(), GenerationConfig(max_new_tokens=2, eos_token_id=3),
                                        _cache(32, block_size=2), 2)
    with pytest.raises(ValueError, match="EOS"):
        s_eos._retire(reqs, None, [])


@pytest.mark.parametrize("chunk", [4, None])
def test_deferred_token_read_keeps_plans_tokens_and_events(chunk, monkeypatch):
    """The deferred path (next forward queued before the sampled values are read, used on CUDA)
    gives the same ragged calls, tokens, events and block accounting as reading them first."""
    from nano_infer_engine_b200.generation import scheduler as sched_mod

    class FakePending(sched_mod._PendingTokens):
        def __init__(self, tokens):  # the values are already on the host here
            self.tokens = tokens.reshape(-1).tolist()

        def values(self):
            return self.tokens

    def run(deferred):
        if deferred:
            original = sched_mod.ContinuousBatchingScheduler._sample

            def sample(self, requests, *, defer=False):
                next_tokens, ids = original(self, requests)
                return (next_tokens, FakePending(next_tokens)) if defer and requests else (next_tokens, ids)

            monkeypatch.setattr(sched_mod.ContinuousBatchingScheduler, "_sample", sample)
        else:
            monkeypatch.undo()
        model = ScriptedModel({"a": (3, 5, 6, 1), "b": (2, 4), "c": (7,)})
        cache = _cache(64, block_size=2)
        s = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=4, prefill_chunk_size=chunk),
                                        cache, 2)
        reqs = [s.add_request(sid, torch.tensor([p])) for sid, p in (("a", [1, 2, 3]), ("b", [4, 5]), ("c", [6]))]
        events = []
        while s.has_work:
            out = s.step()
            events.append((out.token_events, tuple(r.sequence_id for r in out.terminal_requests)))
        seqs = [r.sequence[0].tolist() for r in reqs]
        return seqs, events, model.ragged_calls, model.decode_calls, cache.allocator.allocated_block_count

    sync = run(False)
    deferred = run(True)
    assert deferred == sync


def test_sampler_reads_consecutive_logits_rows_without_a_copy():
    from nano_infer_engine_b200.generation.scheduler import _rows_view

    logits = torch.randn(5, 7)
    view = _rows_view([logits[i] for i in range(5)])
    assert view is not None and view.data_ptr() == logits.data_ptr() and torch.equal(view, logits)
    assert torch.equal(_rows_view([logits[i] for i in range(1, 4)]), logits[1:4])
    assert _rows_view([logits[0], logits[2]]) is None  # a gap
    assert _rows_view([logits[1], logits[0]]) is None  # out of order
    assert _rows_view([logits[0], torch.randn(7)]) is None  # another buffer


def test_prefill_chunks_that_tile_one_buffer_are_passed_without_a_copy():
    from nano_infer_engine_b200.generation.paged_prefill import _flat_view

    tokens = torch.arange(10).view(10, 1)  # a decode step's sampled tokens
    view = _flat_view(tuple(tokens[i : i + 1] for i in range(10)))
    assert view is not None and view.data_ptr() == tokens.data_ptr() and torch.equal(view, torch.arange(10))
    prompt = torch.arange(20).view(1, 20)
    assert torch.equal(_flat_view((prompt[:, 0:5], prompt[:, 5:12], prompt[:, 12:20])), torch.arange(20))
    assert _flat_view((prompt[:, 0:5], prompt[:, 6:12])) is None  # a gap
    assert _flat_view((prompt[:, 5:8], prompt[:, 0:5])) is None  # out of order
    assert _flat_view((tokens[0:1], torch.zeros(1, 1, dtype=torch.long))) is None  # another buffer
