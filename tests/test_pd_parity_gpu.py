"""The in-process P/D drivers against the reference, on one GPU.

``PDContinuousBatchingScheduler`` and ``pd_greedy_generate`` run with both
pools on cuda:0 (the hand-off then runs the block-copy kernel within one
device) on the BASELINE config-1 model in fp32, and must reproduce the golden
that ``tests/golden/make_golden.py --pd`` recorded from the reference's own
P/D scheduler and pd_greedy_generate: every step's token events and terminal
requests, both pools' occupancy after each step, the decode pool's block
table of each request at hand-off, and the final tokens (the smallest greedy
margin in the golden is 6e-4, far above fp32 noise).  The reference's own P/D
unit tests (tests/test_pd_scheduler.py, tests/test_pd_greedy.py) are
re-expressed below on the same device.
"""

import json
from pathlib import Path

import pytest
import torch

import recipes

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "pd_tokens.json").read_text())


def _model(dev):
    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    return build_random_llama(LlamaConfig(**recipes.config1_kwargs()), recipes.CONFIG1_WEIGHT_SEED,
                              recipes.CONFIG1_STD, torch.float32, dev)


def _cache(dev, blocks):
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    return PagedKVCache(blocks, 16, 2, 2, 64, torch.float32, dev)


def _scheduler(dev, config, prefill_blocks, decode_blocks, max_batch):
    from nano_infer_engine_b200.generation.pd_scheduler import PDContinuousBatchingScheduler

    return PDContinuousBatchingScheduler(_model(dev), _model(dev), config, _cache(dev, prefill_blocks),
                                         _cache(dev, decode_blocks), max_batch)


def test_pd_scheduler_matches_reference_golden(cuda):
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.generation.config import GenerationConfig

    want = GOLDEN["scheduler"]
    config = GenerationConfig(max_new_tokens=recipes.PD_NEW_TOKENS, eos_token_id=None)
    sched = _scheduler(cuda, config, recipes.PD_PREFILL_BLOCKS, recipes.PD_DECODE_BLOCKS, recipes.PD_MAX_BATCH)
    prompts = [p.to(cuda) for p in recipes.pd_prompts()]
    reqs = [sched.add_request(f"pd-{i}", p) for i, p in enumerate(prompts)]
    handoff_tables = {}
    admit = sched.decode_scheduler.add_prefilled_request

    def recording_admit(request, last_logits):
        handoff_tables[request.sequence_id] = list(sched.decode_cache.get_block_table(request.sequence_id))
        return admit(request, last_logits)

    sched.decode_scheduler.add_prefilled_request = recording_admit
    steps = []
    with torch.inference_mode():
        while sched.has_work:
            out = sched.step()
            steps.append({
                "events": [[e.sequence_id, e.token_id] for e in out.token_events],
                "terminal": [[r.sequence_id, r.status.name] for r in out.terminal_requests],
                "pending": sched.pending_count,
                "active": sched.active_count,
                "decode_free": sched.decode_cache.allocator.free_block_count,
                "prefill_allocated": sched.prefill_cache.allocator.allocated_block_count,
            })
    ops.check_device_errors(cuda)
    got_tokens = {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs}
    assert got_tokens == want["tokens"]
    assert {r.sequence_id: r.status.name for r in reqs} == want["status"]
    assert handoff_tables == want["handoff_tables"]
    assert len(steps) == len(want["steps"])
    for i, (got, exp) in enumerate(zip(steps, want["steps"])):
        assert got == exp, f"step {i}"
    assert sched.prefill_cache.allocator.allocated_block_count == 0
    assert sched.decode_cache.allocator.allocated_block_count == 0


def test_pd_greedy_matches_reference_golden(cuda):
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.pd_greedy import pd_greedy_generate

    prefill_model, decode_model = _model(cuda), _model(cuda)
    prefill_cache, decode_cache = _cache(cuda, recipes.PD_GREEDY_BLOCKS), _cache(cuda, recipes.PD_GREEDY_BLOCKS)
    prompts = [p.to(cuda) for p in recipes.pd_prompts(recipes.PD_GREEDY_PROMPT_LENS, seed=22)]
    config = GenerationConfig(max_new_tokens=recipes.PD_GREEDY_NEW_TOKENS, eos_token_id=None)
    for i, (p, want) in enumerate(zip(prompts, GOLDEN["greedy"])):
        out = pd_greedy_generate(prefill_model, decode_model, p, config, prefill_cache, decode_cache, f"g-{i}")
        assert out.sequences.device == cuda
        assert out.sequences[0].tolist() == want["sequence"]
        assert out.generated_tokens.tolist() == want["generated"]
        assert out.stopped_by_eos.tolist() == want["stopped_by_eos"]
        assert list(decode_cache.get_block_table(f"g-{i}")) == want["decode_table"]
        assert decode_cache.get_sequence_length(f"g-{i}") == want["decode_length"]
        assert prefill_cache.allocator.allocated_block_count == want["prefill_allocated"] == 0
    want = GOLDEN["greedy_eos"]
    config = GenerationConfig(max_new_tokens=recipes.PD_GREEDY_NEW_TOKENS, eos_token_id=want["eos_token_id"])
    prefill_cache, decode_cache = _cache(cuda, recipes.PD_GREEDY_BLOCKS), _cache(cuda, recipes.PD_GREEDY_BLOCKS)
    out = pd_greedy_generate(prefill_model, decode_model, prompts[0], config, prefill_cache, decode_cache, "g-eos")
    assert out.sequences[0].tolist() == want["sequence"]
    assert out.generated_tokens.tolist() == want["generated"]
    assert out.stopped_by_eos.tolist() == want["stopped_by_eos"] == [True]
    assert list(decode_cache.get_block_table("g-eos")) == want["decode_table"]
    assert decode_cache.get_sequence_length("g-eos") == want["decode_length"]
    ops.check_device_errors(cuda)


# ---- the reference's P/D unit tests, re-expressed on one GPU (config-1 model)
def _short_prompt(cuda, token):
    return torch.tensor([[1, token]], device=cuda)


def test_pd_scheduler_refills_decode_batch_after_a_decode_step(cuda):
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.request import RequestStatus

    sched = _scheduler(cuda, GenerationConfig(max_new_tokens=2, eos_token_id=None), 8, 8, 2)
    reqs = [sched.add_request(f"request-{i}", _short_prompt(cuda, i + 3)) for i in range(3)]
    first = sched.step()
    assert tuple(e.sequence_id for e in first.token_events) == ("request-0", "request-1")
    assert sched.active_count == 2 and sched.pending_count == 1
    second = sched.step()
    assert tuple(e.sequence_id for e in second.token_events) == ("request-0", "request-1")
    assert reqs[0].status is RequestStatus.COMPLETED and reqs[1].status is RequestStatus.COMPLETED
    assert reqs[2].status is RequestStatus.ACTIVE and reqs[2].generated_tokens == 0
    assert sched.active_count == 1 and sched.pending_count == 0
    sched.run_until_idle()
    assert reqs[2].status is RequestStatus.COMPLETED
    assert sched.decode_cache.allocator.allocated_block_count == 0


def test_pd_scheduler_prefill_failure_does_not_block_later_requests(cuda, monkeypatch):
    from nano_infer_engine_b200.generation import pd_handoff
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.request import RequestStatus

    sched = _scheduler(cuda, GenerationConfig(max_new_tokens=1, eos_token_id=None), 8, 8, 2)
    original = pd_handoff.paged_prefill_chunks

    def fail_one_request(model, prompts, cache, sequence_ids):
        if "request-b" in sequence_ids:
            raise RuntimeError("simulated prefill failure")
        return original(model, prompts, cache, sequence_ids)

    monkeypatch.setattr(pd_handoff, "paged_prefill_chunks", fail_one_request)
    reqs = [sched.add_request(s, _short_prompt(cuda, t)) for s, t in (("request-a", 3), ("request-b", 4),
                                                                      ("request-c", 5))]
    sched.run_until_idle()
    assert reqs[0].status is RequestStatus.COMPLETED
    assert reqs[1].status is RequestStatus.FAILED and isinstance(reqs[1].error, RuntimeError)
    assert reqs[2].status is RequestStatus.COMPLETED
    assert sched.prefill_cache.allocator.allocated_block_count == 0
    assert sched.decode_cache.allocator.allocated_block_count == 0


def test_pd_scheduler_close_cancels_pending_and_active_requests(cuda):
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.request import RequestStatus

    sched = _scheduler(cuda, GenerationConfig(max_new_tokens=3, eos_token_id=None), 8, 8, 1)
    active = sched.add_request("request-a", _short_prompt(cuda, 3))
    pending = sched.add_request("request-b", _short_prompt(cuda, 4))
    sched.step()
    assert sched.close() == (pending, active)
    assert active.status is RequestStatus.CANCELLED and pending.status is RequestStatus.CANCELLED
    assert sched.prefill_cache.allocator.allocated_block_count == 0
    assert sched.decode_cache.allocator.allocated_block_count == 0
    assert sched.close() == ()
    with pytest.raises(RuntimeError, match="scheduler is closed"):
        sched.step()


def test_pd_scheduler_rejects_requests_it_cannot_serve(cuda):
    from nano_infer_engine_b200.generation.config import GenerationConfig

    sched = _scheduler(cuda, GenerationConfig(max_new_tokens=3, eos_token_id=None), 2, 2, 2)
    sched.decode_model.config.max_seq_len = 4
    with pytest.raises(ValueError, match="exceeds max model length"):
        sched.add_request("request-a", _short_prompt(cuda, 3))
    sched.decode_model.config.max_seq_len = 4096
    with pytest.raises(ValueError, match="cannot fit in decode cache"):
        sched.add_request("request-b", torch.ones((1, 40), dtype=torch.long, device=cuda))
    sched.add_request("request-c", _short_prompt(cuda, 3))
    with pytest.raises(ValueError, match="already submitted"):
        sched.add_request("request-c", _short_prompt(cuda, 3))
    with pytest.raises(ValueError, match="paged cache device"):
        sched.add_request("request-d", torch.tensor([[1, 2]]))


def test_pd_greedy_releases_both_caches_when_handoff_fails(cuda, monkeypatch):
    from nano_infer_engine_b200.generation import pd_handoff
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.pd_greedy import pd_greedy_generate

    prefill_cache, decode_cache = _cache(cuda, 4), _cache(cuda, 4)

    def fail_after_allocating(source, destination, sequence_id):
        destination.ensure_capacity(sequence_id, 1)
        raise RuntimeError("simulated handoff failure")

    monkeypatch.setattr(pd_handoff, "transfer_sequence", fail_after_allocating)
    with pytest.raises(RuntimeError, match="simulated handoff failure"):
        pd_greedy_generate(_model(cuda), _model(cuda), torch.tensor([[1, 4, 7]], device=cuda),
                           GenerationConfig(max_new_tokens=2), prefill_cache, decode_cache, "request-a")
    assert prefill_cache.allocator.allocated_block_count == 0
    assert decode_cache.allocator.allocated_block_count == 0


def test_pd_greedy_checks_before_any_work(cuda):
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.pd_greedy import pd_greedy_generate

    model = _model(cuda)
    prefill_cache, decode_cache = _cache(cuda, 4), _cache(cuda, 1)
    prompt = torch.tensor([[1, 4, 7]], device=cuda)
    with pytest.raises(ValueError, match="different caches"):
        pd_greedy_generate(model, model, prompt, GenerationConfig(max_new_tokens=2), prefill_cache, prefill_cache)
    with pytest.raises(ValueError, match="not enough free blocks in decode cache"):
        pd_greedy_generate(model, model, prompt, GenerationConfig(max_new_tokens=40), prefill_cache, decode_cache)
    with pytest.raises(ValueError, match="use_cache"):
        pd_greedy_generate(model, model, prompt, GenerationConfig(max_new_tokens=2, use_cache=False),
                           prefill_cache, decode_cache)
    assert prefill_cache.allocator.allocated_block_count == 0
    assert decode_cache.allocator.allocated_block_count == 0


def _all_layers(cache, sid, length):
    pairs = [cache.gather(layer, sid, length) for layer in range(cache.num_layers)]
    return torch.stack([k for k, _ in pairs]), torch.stack([v for _, v in pairs])


class _LoopbackChannel:
    """In-process pair channel: each hand-off is acknowledged at the next poll,
    after the request's KV is copied out of the prefill pool."""

    def __init__(self, cache):
        self.cache = cache
        self.handoffs = {}
        self._acks = []

    def send(self, words):
        from nano_infer_engine_b200.generation.pd_disagg import ACK, HANDOFF

        if words[0] == HANDOFF:
            sid = f"pd-{words[1]}"
            self.handoffs[sid] = (words[3], words[2], *_all_layers(self.cache, sid, words[2]))
            self._acks.append([ACK, words[1]])

    def poll(self, stop_after=None):
        acks, self._acks = self._acks, []
        return acks

    def close(self):
        pass


@pytest.mark.parametrize("chunk_size,budget", [(16, 40), (1, 8), (64, 64)])
def test_chunked_pd_prefill_matches_reference_first_tokens_and_whole_prompt_kv(cuda, chunk_size, budget):
    """run_prefill with chunking: the first token of every request is the reference's (golden), and
    the KV handed off equals a whole-prompt prefill of the same prompt."""
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.generation.paged_prefill import paged_prefill
    from nano_infer_engine_b200.generation.pd_disagg import run_prefill

    model = _model(cuda)
    prompts = [p.to(cuda) for p in recipes.pd_prompts()]
    cache = _cache(cuda, recipes.PD_PREFILL_BLOCKS)
    channel = _LoopbackChannel(cache)
    stats = run_prefill(model, cache, channel, list(enumerate(prompts)), token_budget=budget, chunk_size=chunk_size)
    ops.check_device_errors(cuda)
    assert stats.requests == len(prompts) and stats.tokens == sum(p.shape[1] for p in prompts)
    assert cache.allocator.free_block_count == recipes.PD_PREFILL_BLOCKS
    whole = _cache(cuda, recipes.PD_PREFILL_BLOCKS)
    for i, prompt in enumerate(prompts):
        sid = f"pd-{i}"
        token, length, k, v = channel.handoffs[sid]
        assert length == prompt.shape[1]
        assert token == GOLDEN["scheduler"]["tokens"][sid][0], sid
        with torch.inference_mode():
            paged_prefill(model, (prompt,), whole, (sid,))
        wk, wv = _all_layers(whole, sid, length)
        torch.testing.assert_close(k, wk, atol=1e-4, rtol=0)
        torch.testing.assert_close(v, wv, atol=1e-4, rtol=0)
        whole.release(sid)
