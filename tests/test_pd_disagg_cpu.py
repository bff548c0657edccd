"""P/D disaggregation protocol across two processes (gloo, CPU, scripted models).

Rank 0 prefills and hands requests off; rank 1 imports (host bookkeeping
only here), decodes with continuous batching and acknowledges; the prefill
rank frees each request's blocks on the acknowledgement.  The records travel
through the TCP store (PairChannel) or a pair of named pipes (PipeChannel).
The GPU copy path is exercised by tests/test_pd_gpu.py.
"""

import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nano_infer_engine_b200.generation.config import GenerationConfig
from nano_infer_engine_b200.generation.pd_disagg import (
    ACK,
    DONE,
    HANDOFF,
    HEADER_WORDS,
    PairChannel,
    PipeChannel,
    assign_pairs,
    run_decode,
    run_prefill,
)
from nano_infer_engine_b200.paged_cache import PagedKVCache

PROMPT_LENS = (5, 17, 1, 33, 8, 40)
NEW_TOKENS = 4
PASSES = 3


def _prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 8, (1, n), generator=g) for n in PROMPT_LENS]


def test_router_balances_outstanding_work():
    work = [100, 10, 10, 10, 90, 5]
    assert assign_pairs(work, 2) == [[0, 5], [1, 2, 3, 4]]
    assert assign_pairs(work, 1) == [list(range(6))]
    assert sorted(sum(assign_pairs(work, 3), [])) == list(range(6))


def test_pair_channel_order_and_pass_boundary():
    store = dist.HashStore()
    a = PairChannel(store, 0, 1, HEADER_WORDS)
    b = PairChannel(store, 1, 0, HEADER_WORDS)
    assert b.poll() == []
    for msg in ([1, 7], [3, 1], [1, 8]):
        a.send(msg)
    pad = [0] * (HEADER_WORDS - 2)
    assert b.poll(stop_after=3) == [[1, 7, *pad], [3, 1, *pad]]  # the next pass's record stays queued
    assert b.poll() == [[1, 8, *pad]]
    assert b.poll() == []
    b.send([2, 5])
    assert a.poll() == [[2, 5, *pad]]
    with pytest.raises(ValueError, match="fixed size"):
        a.send([0] * (HEADER_WORDS + 1))


N_PIPE = 256
PIPE_WORDS = 600  # 4800-byte records: larger than the pipe's atomic write size, so writes split


def _pipe_order_worker(rank, port, result_path):
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=60))
    ch = PipeChannel(store, rank, 1 - rank, PIPE_WORDS)
    got = []
    if rank == 0:
        for i in range(N_PIPE):  # 1.2 MB, far more than a pipe holds: the rest waits in the sender's queue
            ch.send([1, i])
        ch.send([3, N_PIPE])
        ch.send([1, N_PIPE + 1])
        ch.close()
        while not got:
            got = ch.poll()
    else:
        import time

        while len(got) < N_PIPE + 1:
            got += ch.poll(stop_after=3)
            time.sleep(0.0005)
        rest = []
        while not rest:
            rest = ch.poll()
        got.append(rest)
        ch.send([2, 9])
        ch.close()
    torch.save(got, f"{result_path}.{rank}")
    store.set(f"done/{rank}", b"1")
    store.wait([f"done/{1 - rank}"])
    ch.release()


def test_pipe_channel_order_backpressure_and_pass_boundary(tmp_path):
    path = str(tmp_path / "pipe")
    mp.start_processes(_pipe_order_worker, args=(_free_port(), path), nprocs=2, start_method="spawn", join=True)
    pad = [0] * (PIPE_WORDS - 2)
    recv = torch.load(path + ".1")
    assert recv[:N_PIPE] == [[1, i, *pad] for i in range(N_PIPE)]
    assert recv[N_PIPE] == [3, N_PIPE, *pad]  # stopped after the pass boundary
    assert recv[N_PIPE + 1] == [[1, N_PIPE + 1, *pad]]  # the next pass's record was kept
    assert torch.load(path + ".0") == [[2, 9, *pad]]


def _worker(rank, port, result_path, kind="store"):
    from test_scheduler_host import ScriptedModel

    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=2, timeout=timedelta(seconds=60))
    prompts = _prompts()
    words = HEADER_WORDS + 16
    channel = (PipeChannel if kind == "pipe" else PairChannel)(store, rank, 1 - rank, words)
    schedules = {f"pd-{i}": tuple(range(1, 8)) for i in range(len(prompts))}
    if rank == 0:
        cache = PagedKVCache(16, 4, 1, 1, 4, torch.float32, "cpu")  # 16 blocks: forces waiting for ACKs
        for _ in range(PASSES):  # passes reuse the channel, the caches and the sequence ids
            first = {}
            stats = run_prefill(ScriptedModel(schedules), cache, channel, list(enumerate(prompts)), token_budget=40,
                                idle_sleep=0.001, first_token_at=first)
        result = {"requests": stats.requests, "batches": stats.batches, "free": cache.allocator.free_block_count,
                  "first": sorted(first)}
    else:
        cache = PagedKVCache(64, 4, 1, 1, 4, torch.float32, "cpu")

        def fake_import(c, sid, length, src_blocks):
            assert len(src_blocks) == -(-length // c.block_size)
            c.ensure_capacity(sid, length)
            c.advance(sid, length)
            return None

        for _ in range(PASSES):
            timings = {}
            reqs = run_decode(ScriptedModel(schedules), cache, channel, lambda i: prompts[i],
                              GenerationConfig(max_new_tokens=NEW_TOKENS), 3, fake_import, 8, idle_sleep=0.001,
                              timings=timings)
        result = {
            "tokens": {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs},
            "status": sorted({r.status.value for r in reqs}),
            "free": cache.allocator.free_block_count,
            "timings": timings,
        }
    torch.save(result, f"{result_path}.{rank}")
    dist.barrier()
    if kind == "pipe":
        channel.release()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("kind", ["store", "pipe"])
def test_prefill_decode_handoff_over_gloo(tmp_path, kind):
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(_free_port(), path, kind), nprocs=2, start_method="spawn", join=True)
    pre = torch.load(path + ".0")
    dec = torch.load(path + ".1")
    assert pre["requests"] == len(PROMPT_LENS)
    assert pre["batches"] > 1  # the 40-token budget splits the prompts
    assert pre["free"] == 16  # every handed-off request was acknowledged and freed
    assert dec["status"] == ["completed"]
    assert dec["free"] == 64
    assert pre["first"] == list(range(len(PROMPT_LENS)))
    assert sorted(dec["timings"]) == list(range(len(PROMPT_LENS)))
    assert all(t1 >= t0 for t0, t1 in dec["timings"].values())
    # first token from the prefill side (its script starts at 1), then the
    # decode side's script continues from its own start for that sequence
    assert len(dec["tokens"]) == len(PROMPT_LENS)
    for toks in dec["tokens"].values():
        assert len(toks) == NEW_TOKENS and toks[0] == 1


def _two_pair_worker(rank, port, result_path):
    """Ranks 2k / 2k+1 form pair k (as bench.py --gpus 4); the router splits the requests."""
    from test_scheduler_host import ScriptedModel

    store = dist.TCPStore("127.0.0.1", port, 4, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=4, timeout=timedelta(seconds=60))
    prompts = _prompts()
    work = [p.shape[1] + NEW_TOKENS for p in prompts]
    mine = assign_pairs(work, 2)[rank // 2]
    channel = PairChannel(store, rank, rank ^ 1, HEADER_WORDS + 16)
    schedules = {f"pd-{i}": tuple(range(1, 8)) for i in range(len(prompts))}
    if rank % 2 == 0:
        cache = PagedKVCache(16, 4, 1, 1, 4, torch.float32, "cpu")
        stats = run_prefill(ScriptedModel(schedules), cache, channel, [(i, prompts[i]) for i in mine],
                            token_budget=24, idle_sleep=0.001)
        result = {"mine": mine, "requests": stats.requests, "free": cache.allocator.free_block_count}
    else:
        cache = PagedKVCache(64, 4, 1, 1, 4, torch.float32, "cpu")

        def fake_import(c, sid, length, src_blocks):
            c.ensure_capacity(sid, length)
            c.advance(sid, length)
            return None

        reqs = run_decode(ScriptedModel(schedules), cache, channel, lambda i: prompts[i],
                          GenerationConfig(max_new_tokens=NEW_TOKENS), 3, fake_import, 8, idle_sleep=0.001)
        result = {"mine": mine, "done": sorted(int(r.sequence_id[3:]) for r in reqs),
                  "status": sorted({r.status.value for r in reqs}), "free": cache.allocator.free_block_count}
    torch.save(result, f"{result_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def test_two_pairs_split_requests_over_four_ranks(tmp_path):
    path = str(tmp_path / "res4")
    mp.start_processes(_two_pair_worker, args=(_free_port(), path), nprocs=4, start_method="spawn", join=True)
    res = [torch.load(f"{path}.{r}") for r in range(4)]
    # both pairs got work, nothing twice, nothing lost
    assert res[0]["mine"] and res[2]["mine"]
    assert sorted(res[0]["mine"] + res[2]["mine"]) == list(range(len(PROMPT_LENS)))
    for pair in (0, 1):
        pre, dec = res[2 * pair], res[2 * pair + 1]
        assert pre["requests"] == len(pre["mine"])
        assert dec["done"] == sorted(pre["mine"])
        assert dec["status"] == ["completed"]
        assert pre["free"] == 16 and dec["free"] == 64


class _LoopbackChannel:
    """In-process stand-in for the pair channel: every hand-off is acknowledged at the next poll."""

    def __init__(self):
        self.sent = []
        self._acks = []

    def send(self, words):
        self.sent.append(list(words))
        if words[0] == HANDOFF:
            self._acks.append([ACK, words[1]])

    def poll(self, stop_after=None):
        acks, self._acks = self._acks, []
        return acks

    def close(self):
        pass


def test_chunked_prefill_plan_budget_order_and_handoffs():
    from test_scheduler_host import ScriptedModel

    prompts = _prompts()
    model = ScriptedModel({f"pd-{i}": tuple(range(1, 20)) for i in range(len(prompts))})
    cache = PagedKVCache(64, 4, 1, 1, 4, torch.float32, "cpu")
    channel = _LoopbackChannel()
    stats = run_prefill(model, cache, channel, list(enumerate(prompts)), token_budget=12, chunk_size=8)
    spans = {}  # sequence -> list of chunk lengths, in call order
    for sids, bounds in model.ragged_calls:
        assert bounds[-1] <= 12  # the token budget holds for every batch
        lengths = [b - a for a, b in zip(bounds, bounds[1:])]
        assert all(0 < n <= 8 for n in lengths)
        for sid, n in zip(sids, lengths):
            spans.setdefault(sid, []).append(n)
    for i, p in enumerate(prompts):
        assert sum(spans[f"pd-{i}"]) == p.shape[1]  # every prompt token prefilled exactly once
    # requests start in arrival order, and a started request is continued in
    # every batch (ahead of new ones) until its last chunk
    firsts = []
    for sids, _ in model.ragged_calls:
        firsts.extend(s for s in sids if s not in firsts)
    assert firsts == [f"pd-{i}" for i in range(len(prompts))]
    left = {f"pd-{i}": p.shape[1] for i, p in enumerate(prompts)}
    for sids, bounds in model.ragged_calls:
        unfinished_before = [s for s in firsts[: firsts.index(sids[-1]) + 1] if 0 < left[s] < prompts[int(s[3:])].shape[1]]
        assert list(sids[: len(unfinished_before)]) == unfinished_before
        for sid, a_, b_ in zip(sids, bounds, bounds[1:]):
            left[sid] -= b_ - a_
    handoffs = [m for m in channel.sent if m[0] == HANDOFF]
    assert sorted(m[1] for m in handoffs) == list(range(len(prompts)))
    for m in handoffs:
        index, length, token, nblk = m[1], m[2], m[3], m[4]
        assert length == prompts[index].shape[1] and nblk == -(-length // 4)
        assert token == len(spans[f"pd-{index}"])  # the scripted token of the request's last chunk
    assert channel.sent[-1][0] == DONE and stats.requests == len(prompts)
    assert stats.tokens == sum(p.shape[1] for p in prompts)
    assert cache.allocator.free_block_count == 64  # every hand-off acknowledged and freed


def test_chunked_prefill_starts_a_request_only_when_its_whole_prompt_fits():
    from test_scheduler_host import ScriptedModel

    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 8, (1, n), generator=g) for n in (40, 40, 6)]
    model = ScriptedModel()
    cache = PagedKVCache(12, 4, 1, 1, 4, torch.float32, "cpu")  # 48 tokens: one 40-token prompt at a time
    channel = _LoopbackChannel()
    stats = run_prefill(model, cache, channel, list(enumerate(prompts)), token_budget=16, chunk_size=8)
    assert stats.requests == 3 and cache.allocator.free_block_count == 12
    # request 1 may not start before request 0 is handed off and its blocks are back
    first_call_of_1 = next(n for n, (sids, _) in enumerate(model.ragged_calls) if "pd-1" in sids)
    last_call_of_0 = max(n for n, (sids, _) in enumerate(model.ragged_calls) if "pd-0" in sids)
    assert first_call_of_1 > last_call_of_0


def test_chunk_size_must_be_positive():
    with pytest.raises(ValueError, match="chunk_size"):
        run_prefill(None, PagedKVCache(4, 4, 1, 1, 4, torch.float32, "cpu"), _LoopbackChannel(), [], chunk_size=0)


def _group_worker(rank, port, result_path):
    """One prefill rank (0) feeding two decode ranks (1, 2) over pipes: a 1:2 P:D group."""
    from test_scheduler_host import ScriptedModel

    from nano_infer_engine_b200.generation.pd_disagg import assign_groups

    store = dist.TCPStore("127.0.0.1", port, 3, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=3, timeout=timedelta(seconds=60))
    prompts = _prompts()
    work = [p.shape[1] + NEW_TOKENS for p in prompts]
    (slots,) = assign_groups(work, 1, 2)
    schedules = {f"pd-{i}": tuple(range(1, 8)) for i in range(len(prompts))}
    words = HEADER_WORDS + 16
    if rank == 0:
        channels = [PipeChannel(store, 0, peer, words) for peer in (1, 2)]
        mine = sorted(slots[0] + slots[1])
        route = [0 if i in slots[0] else 1 for i in mine]
        cache = PagedKVCache(16, 4, 1, 1, 4, torch.float32, "cpu")
        stats = run_prefill(ScriptedModel(schedules), cache, channels, [(i, prompts[i]) for i in mine],
                            token_budget=24, chunk_size=8, route=route, idle_sleep=0.001)
        result = {"requests": stats.requests, "free": cache.allocator.free_block_count}
    else:
        channels = [PipeChannel(store, rank, 0, words)]
        cache = PagedKVCache(64, 4, 1, 1, 4, torch.float32, "cpu")

        def fake_import(c, sid, length, src_blocks):
            c.ensure_capacity(sid, length)
            c.advance(sid, length)
            return None

        reqs = run_decode(ScriptedModel(schedules), cache, channels[0], lambda i: prompts[i],
                          GenerationConfig(max_new_tokens=NEW_TOKENS), 4, fake_import, 8, idle_sleep=0.001)
        result = {"done": sorted(int(r.sequence_id[3:]) for r in reqs), "mine": sorted(slots[rank - 1]),
                  "status": sorted({r.status.value for r in reqs}), "free": cache.allocator.free_block_count}
    torch.save(result, f"{result_path}.{rank}")
    dist.barrier()
    for ch in channels:
        ch.release()
    dist.destroy_process_group()


def test_one_prefill_rank_feeds_two_decode_ranks(tmp_path):
    path = str(tmp_path / "grp")
    mp.start_processes(_group_worker, args=(_free_port(), path), nprocs=3, start_method="spawn", join=True)
    pre, d1, d2 = (torch.load(f"{path}.{r}") for r in range(3))
    assert pre["requests"] == len(PROMPT_LENS) and pre["free"] == 16
    assert d1["done"] == d1["mine"] and d2["done"] == d2["mine"]  # each decode rank got its routed requests
    assert d1["mine"] and d2["mine"] and sorted(d1["mine"] + d2["mine"]) == list(range(len(PROMPT_LENS)))
    assert d1["status"] == d2["status"] == ["completed"] and d1["free"] == d2["free"] == 64


def test_group_router_gives_each_decode_rank_one_copy_of_a_replicated_job():
    from nano_infer_engine_b200.generation.pd_disagg import assign_groups

    base = [7, 30, 3, 12]
    for groups, k in ((1, 3), (2, 3), (2, 1)):
        copies = groups * k
        job = [w for w in base for _ in range(copies)]  # copies of each request, interleaved
        out = assign_groups(job, groups, k)
        assert len(out) == groups and all(len(g) == k for g in out)
        for group in out:
            for slot in group:
                assert sorted(job[i] for i in slot) == sorted(base)


def test_run_prefill_route_is_checked_before_any_work():
    cache = PagedKVCache(8, 4, 1, 1, 4, torch.float32, "cpu")
    prompts = [(0, torch.zeros(1, 3, dtype=torch.long)), (1, torch.zeros(1, 2, dtype=torch.long))]
    with pytest.raises(ValueError, match="route is required"):
        run_prefill(None, cache, [_LoopbackChannel(), _LoopbackChannel()], prompts)
    with pytest.raises(ValueError, match="route must name"):
        run_prefill(None, cache, [_LoopbackChannel(), _LoopbackChannel()], prompts, route=[0, 2])
    with pytest.raises(ValueError, match="route must name"):
        run_prefill(None, cache, [_LoopbackChannel(), _LoopbackChannel()], prompts, route=[0])
    assert cache.allocator.free_block_count == 8


def test_assign_groups_with_one_decode_rank_is_the_pair_router():
    from nano_infer_engine_b200.generation.pd_disagg import assign_groups

    rng = torch.Generator().manual_seed(3)
    work = torch.randint(1, 500, (57,), generator=rng).tolist()
    for groups in (1, 2, 3, 5):
        assert [g[0] for g in assign_groups(work, groups, 1)] == assign_pairs(work, groups)
