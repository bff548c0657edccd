"""Generate the golden fixtures by running the REFERENCE implementation.

Run where the reference checkout is available, with NIE_REFERENCE_SRC set
to its `src` directory (the one holding the `nano_infer_engine` package):

    NIE_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

It imports the reference package ``nano_infer_engine``, this repository's
seeded recipes (tests/golden/recipes.py) and the oracle's seeded weight
recipe (oracle/weights.py; nothing from the product package), and writes only
reference OUTPUTS: paging.json, decode_<case>.pt, ragged_<case>.pt,
config1_tokens.json, pd_tokens.json (``--pd``) and config2_greedy256.json
(``--config2-dense``).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent.parent))
if "NIE_REFERENCE_SRC" not in os.environ:
    raise SystemExit("set NIE_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["NIE_REFERENCE_SRC"])

import recipes  # noqa: E402
from nano_infer_engine.generation.config import GenerationConfig  # noqa: E402
from nano_infer_engine.generation.scheduler import ContinuousBatchingScheduler  # noqa: E402
from nano_infer_engine.layers.attention import GroupedQueryAttention  # noqa: E402
from nano_infer_engine.layers.paged_attention import batched_paged_attention_reference  # noqa: E402
from nano_infer_engine.layers.rope import Rope  # noqa: E402
from nano_infer_engine.models.llama import Llama3_2, LlamaConfig  # noqa: E402
from nano_infer_engine.paged_cache import PagedKVCache  # noqa: E402

from oracle.weights import LLAMA_1B, random_llama_state  # noqa: E402


def _reference_llama(kwargs: dict, seed: int, std: float, dtype: torch.dtype, **extra) -> Llama3_2:
    """The reference's Llama3_2 holding the seeded random-init weights."""
    model = Llama3_2(LlamaConfig(**kwargs, **extra)).to(dtype).eval()
    model.load_state_dict(random_llama_state(kwargs, seed, std, dtype))
    return model


def paging() -> dict:
    cache = PagedKVCache(32, 16, 1, 1, 16, torch.float32, "cpu")
    trace = []
    for op in recipes.paging_scenario():
        kind, sid = op[0], op[1]
        if kind == "ensure":
            cache.ensure_capacity(sid, op[2])
        elif kind == "advance":
            cache.advance(sid, op[2])
        elif kind == "release":
            cache.release(sid)
        trace.append({
            "op": list(op),
            "tables": {s: list(cache.get_block_table(s)) for s in sorted(cache._block_tables)},
            "lengths": {s: cache.get_sequence_length(s) for s in sorted(cache._block_tables)},
            "free": cache.allocator.free_block_count,
        })
    # ragged metadata of one step over the surviving sequences, via the
    # reference's own position -> (block, offset) resolution
    ids = sorted(cache._block_tables)
    contexts = [cache.get_sequence_length(s) for s in ids]
    qlens = [min(3, len(cache.get_block_table(s)) * 16 - c) for s, c in zip(ids, contexts)]
    slots = []
    for s, c, q in zip(ids, contexts, qlens):
        for j in range(q):
            block, off = cache._resolve_position(s, c + j)
            slots.append(block * 16 + off)
    return {"trace": trace, "step": {"ids": ids, "contexts": contexts, "qlens": qlens, "slots": slots}}


def decode(name: str) -> dict:
    case = recipes.decode_case(name)
    out = batched_paged_attention_reference(
        case["query"], case["key_cache"], case["value_cache"],
        tuple(tuple(t) for t in case["tables"]), tuple(case["seq_lens"]), case["layer"],
    )
    return {"out": out}


def ragged(name: str) -> dict:
    c = recipes.ragged_case(name)
    attn = GroupedQueryAttention(c["hq"], c["hkv"], c["hidden"], Rope(64, c["rope_theta"])).to(c["dtype"])
    attn.load_state_dict(c["weights"])
    cache = PagedKVCache(c["num_blocks"], c["block_size"], 1, c["hkv"], 64, c["dtype"], "cpu")
    for sid, n in c["warmup"]:
        cache.ensure_capacity(sid, n)
    for sid in c["release"]:
        cache.release(sid)
    for sid, ctx, (hk, hv), ql in zip(c["ids"], c["contexts"], c["history"], c["qlens"]):
        cache.ensure_capacity(sid, ctx + ql)
        if ctx:
            cache.write(0, sid, 0, hk, hv)
            cache.advance(sid, ctx)
    qsl = torch.tensor([0] + torch.tensor(c["qlens"]).cumsum(0).tolist())
    with torch.inference_mode():
        out = attn.forward_ragged(c["x"], paged_cache=cache, layer_index=0, sequence_ids=c["ids"],
                                  query_start_loc=qsl, context_lengths=tuple(c["contexts"]))
    tables = {s: list(cache.get_block_table(s)) for s in c["ids"]}
    keys = {s: cache.gather(0, s, ctx + ql)[0] for s, ctx, ql in zip(c["ids"], c["contexts"], c["qlens"])}
    values = {s: cache.gather(0, s, ctx + ql)[1] for s, ctx, ql in zip(c["ids"], c["contexts"], c["qlens"])}
    return {"out": out, "tables": tables, "keys": keys, "values": values}


def config1() -> dict:
    model = _reference_llama(recipes.config1_kwargs(), recipes.CONFIG1_WEIGHT_SEED, recipes.CONFIG1_STD,
                             torch.float32)
    cache = PagedKVCache(64, 16, 2, 2, 64, torch.float32, "cpu")
    config = GenerationConfig(max_new_tokens=16, prefill_chunk_size=32)
    sched = ContinuousBatchingScheduler(model, config, cache, 4)
    prompts = recipes.config1_prompts()
    ids = [f"req-{i}" for i in range(len(prompts))]
    reqs = [sched.add_request(s, p) for s, p in zip(ids, prompts)]
    margins: dict[str, list[float]] = {s: [] for s in ids}
    steps = []
    original = model.forward_ragged

    def recording(input_ids, *, kv_cache, sequence_ids, query_start_loc):
        steps.append({"ids": list(sequence_ids), "qsl": query_start_loc.tolist(),
                      "tables": {s: list(kv_cache.get_block_table(s)) for s in sequence_ids if s in kv_cache._block_tables}})
        logits = original(input_ids, kv_cache=kv_cache, sequence_ids=sequence_ids, query_start_loc=query_start_loc)
        for s, e in zip(sequence_ids, query_start_loc.tolist()[1:]):
            top2 = logits[e - 1].topk(2).values
            margins[s].append(float(top2[0] - top2[1]))
        steps[-1]["tables_after"] = {s: list(kv_cache.get_block_table(s)) for s in sequence_ids}
        return logits

    model.forward_ragged = recording
    with torch.inference_mode():
        sched.run_until_idle()
    return {
        "tokens": {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs},
        "margins": margins,
        "steps": steps,
        "free_blocks_after": cache.allocator.free_block_count,
    }


def pd_pipeline() -> dict:
    """The reference's PDContinuousBatchingScheduler and pd_greedy_generate on the
    config-1 model (fp32, both caches on the host): every step's token events and
    terminal requests, the decode pool's block table of each request at hand-off,
    both pools' occupancy after each step, and the greedy margins."""
    from nano_infer_engine.generation.pd_greedy import pd_greedy_generate
    from nano_infer_engine.generation.pd_scheduler import PDContinuousBatchingScheduler

    kwargs = recipes.config1_kwargs()

    def model():
        return _reference_llama(kwargs, recipes.CONFIG1_WEIGHT_SEED, recipes.CONFIG1_STD, torch.float32)

    def cache(blocks):
        return PagedKVCache(blocks, 16, 2, 2, 64, torch.float32, "cpu")

    config = GenerationConfig(max_new_tokens=recipes.PD_NEW_TOKENS, eos_token_id=None)
    sched = PDContinuousBatchingScheduler(model(), model(), config, cache(recipes.PD_PREFILL_BLOCKS),
                                          cache(recipes.PD_DECODE_BLOCKS), recipes.PD_MAX_BATCH)
    prompts = recipes.pd_prompts()
    ids = [f"pd-{i}" for i in range(len(prompts))]
    reqs = [sched.add_request(s, p) for s, p in zip(ids, prompts)]
    handoff_tables: dict[str, list[int]] = {}
    admit = sched.decode_scheduler.add_prefilled_request

    def recording_admit(request, last_logits):
        handoff_tables[request.sequence_id] = list(sched.decode_cache.get_block_table(request.sequence_id))
        return admit(request, last_logits)

    sched.decode_scheduler.add_prefilled_request = recording_admit
    margins: dict[str, list[float]] = {s: [] for s in ids}
    decode_step = sched.decode_scheduler.step

    def recording_step():
        for r in sched.decode_scheduler.active_requests:
            top2 = r.last_logits.float().topk(2).values
            margins[r.sequence_id].append(float(top2[0] - top2[1]))
        return decode_step()

    sched.decode_scheduler.step = recording_step
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
    scheduler_out = {
        "tokens": {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs},
        "status": {r.sequence_id: r.status.name for r in reqs},
        "handoff_tables": handoff_tables,
        "steps": steps,
        "margins": margins,
    }

    # pd_greedy_generate: two requests in a row through the same caches (the
    # decode pool keeps each finished sequence), then one stopped by EOS
    greedy = []
    prefill_model, decode_model = model(), model()
    prefill_cache, decode_cache = cache(recipes.PD_GREEDY_BLOCKS), cache(recipes.PD_GREEDY_BLOCKS)
    gprompts = recipes.pd_prompts(recipes.PD_GREEDY_PROMPT_LENS, seed=22)
    gconfig = GenerationConfig(max_new_tokens=recipes.PD_GREEDY_NEW_TOKENS, eos_token_id=None)
    for i, p in enumerate(gprompts):
        out = pd_greedy_generate(prefill_model, decode_model, p, gconfig, prefill_cache, decode_cache, f"g-{i}")
        greedy.append({
            "sequence": out.sequences[0].tolist(),
            "generated": out.generated_tokens.tolist(),
            "stopped_by_eos": out.stopped_by_eos.tolist(),
            "decode_table": list(decode_cache.get_block_table(f"g-{i}")),
            "decode_length": decode_cache.get_sequence_length(f"g-{i}"),
            "prefill_allocated": prefill_cache.allocator.allocated_block_count,
        })
    eos = greedy[0]["sequence"][gprompts[0].shape[1] + recipes.PD_GREEDY_EOS_INDEX]
    econfig = GenerationConfig(max_new_tokens=recipes.PD_GREEDY_NEW_TOKENS, eos_token_id=eos)
    prefill_cache, decode_cache = cache(recipes.PD_GREEDY_BLOCKS), cache(recipes.PD_GREEDY_BLOCKS)
    out = pd_greedy_generate(prefill_model, decode_model, gprompts[0], econfig, prefill_cache, decode_cache, "g-eos")
    eos_out = {
        "eos_token_id": eos,
        "sequence": out.sequences[0].tolist(),
        "generated": out.generated_tokens.tolist(),
        "stopped_by_eos": out.stopped_by_eos.tolist(),
        "decode_table": list(decode_cache.get_block_table("g-eos")),
        "decode_length": decode_cache.get_sequence_length("g-eos"),
    }
    return {"scheduler": scheduler_out, "greedy": greedy, "greedy_eos": eos_out}


def config2_dense() -> dict:
    """BASELINE config 2 in full: the 16 seeded prompts, 256 greedy tokens each, bf16,
    through the reference's dense greedy_generate (generation/greedy.py:10-122), one
    request at a time (no padding), with the top-1 minus top-2 logit margin of every
    greedy decision.  The reference pins this path equal to its paged scheduler
    (tests/test_paged_greedy_generation.py:145-200); its paged path would take hours
    here because of the per-token Python gather loops."""
    from nano_infer_engine.generation.greedy import greedy_generate

    torch.set_num_threads(os.cpu_count() or 1)
    model = _reference_llama(LLAMA_1B, recipes.CONFIG2_WEIGHT_SEED, 0.02, torch.bfloat16, max_seq_len=29600)
    config = GenerationConfig(max_new_tokens=recipes.CONFIG2_FULL_NEW_TOKENS, eos_token_id=None)
    forward = model.forward
    margins: list[float] = []

    def recording(*args, **kwargs):
        logits = forward(*args, **kwargs)
        top2 = logits[0, -1].float().topk(2).values
        margins.append(float(top2[0] - top2[1]))
        return logits

    model.forward = recording
    out_tokens, out_margins = {}, {}
    for i, prompt in enumerate(recipes.config2_prompts()):
        margins.clear()
        out = greedy_generate(model, prompt, config)
        out_tokens[f"req-{i}"] = out.sequences[0, prompt.shape[1]:].tolist()
        out_margins[f"req-{i}"] = list(margins)
        print(f"config2 dense: request {i} ({prompt.shape[1]} prompt tokens) done", flush=True)
    return {"new_tokens": recipes.CONFIG2_FULL_NEW_TOKENS, "tokens": out_tokens, "margins": out_margins}


def main() -> None:
    if "--config2-dense" in sys.argv:
        (HERE / "config2_greedy256.json").write_text(json.dumps(config2_dense()))
        print("config2 dense golden written")
        return
    if "--pd" in sys.argv:
        (HERE / "pd_tokens.json").write_text(json.dumps(pd_pipeline()))
        print("pd golden written")
        return
    (HERE / "paging.json").write_text(json.dumps(paging(), indent=1))
    for name in recipes.DECODE_CASES:
        torch.save(decode(name), HERE / f"decode_{name}.pt")
    for name in recipes.RAGGED_CASES:
        torch.save(ragged(name), HERE / f"ragged_{name}.pt")
    (HERE / "config1_tokens.json").write_text(json.dumps(config1()))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
