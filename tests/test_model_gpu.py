"""Model-level parity on the GPU against fixtures produced by the reference.

* GroupedQueryAttention.forward_ragged (projections, RoPE, slot write,
  decode + varlen attention, o_proj) on a mixed prefill/decode step;
* BASELINE config 1 (tiny fp32 Llama) end to end through the chunked
  continuous-batching scheduler: greedy tokens, per-step ragged call
  (sequence order, query_start_loc) and block tables must all match.
"""

import json
from pathlib import Path

import pytest
import torch

import recipes

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", recipes.RAGGED_CASES)
def test_gqa_forward_ragged_matches_reference(cuda, name):
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.layers.attention import GroupedQueryAttention
    from nano_infer_engine_b200.layers.rope import Rope
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    c = recipes.ragged_case(name)
    golden = torch.load(GOLDEN / f"ragged_{name}.pt")
    attn = GroupedQueryAttention(c["hq"], c["hkv"], c["hidden"], Rope(64, c["rope_theta"])).to(c["dtype"])
    attn.load_state_dict(c["weights"])
    attn = attn.to(cuda)
    cache = PagedKVCache(c["num_blocks"], c["block_size"], 1, c["hkv"], 64, c["dtype"], cuda)
    for sid, n in c["warmup"]:
        cache.ensure_capacity(sid, n)
    for sid in c["release"]:
        cache.release(sid)
    for sid, ctx, (hk, hv), ql in zip(c["ids"], c["contexts"], c["history"], c["qlens"]):
        cache.ensure_capacity(sid, ctx + ql)
        if ctx:
            cache.write(0, sid, 0, hk.to(cuda), hv.to(cuda))
            cache.advance(sid, ctx)
    qsl = torch.tensor([0] + torch.tensor(c["qlens"]).cumsum(0).tolist(), device=cuda)
    with torch.inference_mode():
        out = attn.forward_ragged(c["x"].to(cuda), paged_cache=cache, layer_index=0, sequence_ids=c["ids"],
                                  query_start_loc=qsl, context_lengths=tuple(c["contexts"]))
    ops.check_device_errors(cuda)
    for sid, ctx, ql in zip(c["ids"], c["contexts"], c["qlens"]):
        assert list(cache.get_block_table(sid)) == golden["tables"][sid]
        k, v = cache.gather(0, sid, ctx + ql)
        # K after RoPE and V are projections of the same x: bitwise equal is
        # not guaranteed across devices, so compare at the dtype's ulp scale
        tol = 1e-2 if c["dtype"] == torch.bfloat16 else 1e-5
        torch.testing.assert_close(k.cpu().float(), golden["keys"][sid].float(), atol=tol, rtol=tol)
        torch.testing.assert_close(v.cpu().float(), golden["values"][sid].float(), atol=tol, rtol=tol)
    tol = 2e-2 if c["dtype"] == torch.bfloat16 else 1e-4
    torch.testing.assert_close(out.cpu().float(), golden["out"].float(), atol=tol, rtol=0)


def test_config1_greedy_tokens_and_step_plan_match_reference(cuda):
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
    from nano_infer_engine_b200.models.llama import Llama3_2, LlamaConfig, init_random_weights_
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    golden = json.loads((GOLDEN / "config1_tokens.json").read_text())
    model = Llama3_2(LlamaConfig(**recipes.config1_kwargs())).eval()
    init_random_weights_(model, recipes.CONFIG1_WEIGHT_SEED, recipes.CONFIG1_STD)
    model = model.to(cuda)
    cache = PagedKVCache(64, 16, 2, 2, 64, torch.float32, cuda)
    sched = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=16, prefill_chunk_size=32), cache, 4)
    prompts = [p.to(cuda) for p in recipes.config1_prompts()]
    ids = [f"req-{i}" for i in range(len(prompts))]
    reqs = [sched.add_request(s, p) for s, p in zip(ids, prompts)]
    steps = []
    original = model.forward_ragged

    def recording(input_ids, *, kv_cache, sequence_ids, query_start_loc):
        logits = original(input_ids, kv_cache=kv_cache, sequence_ids=sequence_ids, query_start_loc=query_start_loc)
        steps.append({"ids": list(sequence_ids), "qsl": query_start_loc.tolist(),
                      "tables_after": {s: list(kv_cache.get_block_table(s)) for s in sequence_ids}})
        return logits

    model.forward_ragged = recording
    with torch.inference_mode():
        sched.run_until_idle()
    tokens = {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs}
    assert tokens == golden["tokens"]
    assert len(steps) == len(golden["steps"])
    for got, want in zip(steps, golden["steps"]):
        assert got["ids"] == want["ids"]
        assert got["qsl"] == want["qsl"]
        assert got["tables_after"] == want["tables_after"]
    assert cache.allocator.free_block_count == golden["free_blocks_after"]


def _llama_shaped_model(cuda, seed=7):
    """Llama attention geometry (head_dim 64, 4 q heads per kv head, bf16) at small width."""
    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    cfg = LlamaConfig(vocab_size=512, hidden_size=512, mlp_inner_size=1024, num_layers=2, q_head_num=8,
                      kv_head_num=2, max_seq_len=4096)
    return build_random_llama(cfg, seed, 0.02, torch.bfloat16, cuda), cfg


def _generate(model, cfg, prompts, cuda, *, graphs, chunk):
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    model.cuda_graphs = graphs
    dtype = model.embed.weight.dtype
    cache = PagedKVCache(256, 16, cfg.num_layers, cfg.kv_head_num, cfg.head_dim, dtype, cuda)
    config = GenerationConfig(max_new_tokens=12, prefill_chunk_size=chunk, max_prefill_tokens_per_step=64 if chunk else None)
    sched = ContinuousBatchingScheduler(model, config, cache, 4)
    reqs = [sched.add_request(f"r{i}", p) for i, p in enumerate(prompts)]
    logits = []
    with torch.inference_mode():
        while sched.has_work:
            sched.step()
            logits.extend(r.last_logits.float().cpu() for r in sched.active_requests if r.last_logits is not None)
    # the scheduler marks a request FAILED (instead of raising) when its step throws
    assert [(r.status.value, r.error) for r in reqs] == [("completed", None)] * len(reqs)
    assert all(r.generated_tokens == config.max_new_tokens for r in reqs)
    return [r.sequence[0].tolist() for r in reqs], logits, cache


def test_precaptured_decode_graphs_match_eager_and_no_step_captures(cuda, monkeypatch):
    """Graphs captured ahead (table reserved first) serve every later decode step: same tokens as eager."""
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
    from nano_infer_engine_b200.models import llama
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    model, cfg = _llama_shaped_model(cuda)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (1, n), generator=g).to(cuda) for n in (9, 33, 70, 18)]
    eager_tokens, _, _ = _generate(model, cfg, prompts, cuda, graphs=False, chunk=None)

    model.cuda_graphs = True
    cache = PagedKVCache(256, 16, cfg.num_layers, cfg.kv_head_num, cfg.head_dim, torch.bfloat16, cuda)
    sched = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=12), cache, 4)
    reqs = [sched.add_request(f"r{i}", p) for i, p in enumerate(prompts)]
    captured = []
    original = llama._DecodeGraph.__init__

    def counting(self, *args):
        captured.append(args[-1])
        original(self, *args)

    monkeypatch.setattr(llama._DecodeGraph, "__init__", counting)
    with torch.inference_mode():
        sched.step()  # the first step initialises the library handles
        cache.reserve_table(8, -(-cfg.max_seq_len // 16))
        assert model.capture_decode_graphs(cache, range(1, 5)) == 4
        assert model.capture_decode_graphs(cache, range(1, 5)) == 0  # already held
        captured.clear()
        while sched.has_work:
            sched.step()
    ops.check_device_errors(cuda)
    assert captured == [], f"decode steps captured graphs mid-run: {captured}"
    assert [r.sequence[0].tolist() for r in reqs] == eager_tokens


@pytest.mark.parametrize("chunk", [32, None])
def test_cuda_graph_decode_matches_eager(cuda, chunk):
    """Decode steps replayed from CUDA graphs give the eager path's tokens and logits."""
    from nano_infer_engine_b200 import ops

    model, cfg = _llama_shaped_model(cuda)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (1, n), generator=g).to(cuda) for n in (5, 40, 77, 16, 130)]
    eager_tokens, eager_logits, _ = _generate(model, cfg, prompts, cuda, graphs=False, chunk=chunk)
    graph_tokens, graph_logits, cache = _generate(model, cfg, prompts, cuda, graphs=True, chunk=chunk)
    ops.check_device_errors(cuda)
    assert graph_tokens == eager_tokens
    assert len(graph_logits) == len(eager_logits)
    for a, b in zip(graph_logits, eager_logits):
        torch.testing.assert_close(a, b, atol=1e-2, rtol=0)
    assert getattr(cache, "_decode_graphs", None), "no decode step was captured"
    assert cache.allocator.allocated_block_count == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_native_layer_loop_matches_python_loop(cuda, dtype):
    """The C++ layer loop issues the Python loop's kernels and GEMMs: identical logits, bit for bit."""
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    assert ops.layer_loop_ext() is not None, "the layer-loop extension was not built"
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, mlp_inner_size=1024, num_layers=3, q_head_num=8,
                      kv_head_num=2, max_seq_len=4096)
    model = build_random_llama(cfg, 11, 0.02, dtype, cuda)
    model._ensure_fused()
    assert model._layer_loop_args(dtype) is not None
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (1, n), generator=g).to(cuda) for n in (3, 45, 130, 16)]
    results = []
    for native in (False, True):
        model.native_layer_loop = native
        results.append(_generate(model, cfg, prompts, cuda, graphs=False, chunk=32))
    ops.check_device_errors(cuda)
    (py_tokens, py_logits, _), (cc_tokens, cc_logits, cache) = results
    assert cc_tokens == py_tokens
    assert len(cc_logits) == len(py_logits)
    for a, b in zip(cc_logits, py_logits):
        assert torch.equal(a, b)
    assert cache.allocator.allocated_block_count == 0


@pytest.mark.parametrize("chunk", [32, None])
def test_eos_schedule_matches_eos_free_run_until_each_stop(cuda, chunk):
    """With an EOS token the scheduler reads each step's tokens before queuing the next
    forward (synchronous path); without one it queues first (deferred path).  Both must
    produce the same tokens up to each request's first EOS, where it stops."""
    model, cfg = _llama_shaped_model(cuda, seed=13)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (1, n), generator=g).to(cuda) for n in (6, 50, 21)]
    free_tokens, _, _ = _generate(model, cfg, prompts, cuda, graphs=True, chunk=chunk)
    first = free_tokens[0][prompts[0].shape[1]:]
    eos = first[2]  # request 0 stops after three tokens

    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    cache = PagedKVCache(256, 16, cfg.num_layers, cfg.kv_head_num, cfg.head_dim, torch.bfloat16, cuda)
    config = GenerationConfig(max_new_tokens=12, eos_token_id=eos, prefill_chunk_size=chunk,
                              max_prefill_tokens_per_step=64 if chunk else None)
    sched = ContinuousBatchingScheduler(model, config, cache, 4)
    reqs = [sched.add_request(f"r{i}", p) for i, p in enumerate(prompts)]
    with torch.inference_mode():
        sched.run_until_idle()
    for r, free, p in zip(reqs, free_tokens, prompts):
        got = r.sequence[0, p.shape[1]:].tolist()
        want = free[p.shape[1]:]
        stop = want.index(eos) + 1 if eos in want else len(want)
        assert got == want[:stop]
        assert r.status.value == "completed" and r.finished == (eos in want)
    assert cache.allocator.allocated_block_count == 0
