"""Generate the golden fixtures by running the REFERENCE implementation.

Run where the reference checkout is available, with NIE_REFERENCE_SRC set
to its `src` directory (the one holding the `nano_infer_engine` package):

    NIE_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

It imports the reference package ``nano_infer_engine`` and this repository's
seeded recipes (tests/golden/recipes.py) and writes only reference OUTPUTS:
paging.json, decode_<case>.pt, ragged_<case>.pt, config1_tokens.json.
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

from nano_infer_engine_b200.models.llama import init_random_weights_  # noqa: E402


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
    torch.manual_seed(0)
    model = Llama3_2(LlamaConfig(**recipes.config1_kwargs())).eval()
    init_random_weights_(model, recipes.CONFIG1_WEIGHT_SEED, recipes.CONFIG1_STD)
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


def config2_reduced() -> dict:
    """BASELINE config 2 (Llama-3.2-1B shape, bf16, random init std 0.02) with the
    bench's seeded workload but only CONFIG2_NEW_TOKENS new tokens per request."""
    from nano_infer_engine_b200.models.llama import LlamaConfig as OurConfig, build_random_llama

    ours = build_random_llama(OurConfig(max_seq_len=29600), recipes.CONFIG2_WEIGHT_SEED, 0.02, torch.bfloat16, "cpu")
    model = Llama3_2(LlamaConfig(max_seq_len=29600)).to(torch.bfloat16).eval()
    model.load_state_dict(ours.state_dict())
    del ours
    prompts = recipes.config2_prompts()
    blocks = sum((p.shape[1] + recipes.CONFIG2_NEW_TOKENS + 15) // 16 for p in prompts) + 16
    cache = PagedKVCache(blocks, 16, 16, 8, 64, torch.bfloat16, "cpu")
    config = GenerationConfig(max_new_tokens=recipes.CONFIG2_NEW_TOKENS, prefill_chunk_size=128,
                              max_prefill_tokens_per_step=512)
    sched = ContinuousBatchingScheduler(model, config, cache, len(prompts))
    ids = [f"req-{i}" for i in range(len(prompts))]
    reqs = [sched.add_request(s, p) for s, p in zip(ids, prompts)]
    # margin (top-1 minus top-2 logit) of every greedy decision, read from the
    # logits each active request holds right before the step that samples it
    margins: dict[str, list[float]] = {s: [] for s in ids}
    with torch.inference_mode():
        while sched.has_work:
            for r in sched.active_requests:
                top2 = r.last_logits.float().topk(2).values
                margins[r.sequence_id].append(float(top2[0] - top2[1]))
            sched.step()
    return {
        "tokens": {r.sequence_id: r.sequence[0, r.prompt.shape[1]:].tolist() for r in reqs},
        "margins": margins,
    }


def main() -> None:
    if "--config2" in sys.argv:
        (HERE / "config2_tokens.json").write_text(json.dumps(config2_reduced()))
        print("config2 golden written")
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
