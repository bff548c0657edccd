"""Pin the CPU oracle against fixtures produced by the reference itself (tests/golden)."""

import json
from pathlib import Path

import pytest
import torch

import recipes
from oracle import attention as oatt
from oracle.engine import OracleCache, inv_freq, rope
from oracle.paging import OracleTables, ragged_metadata

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_paging_trace_matches_reference():
    golden = json.loads((GOLDEN / "paging.json").read_text())
    tables = OracleTables(32, 16)
    for op, expected in zip(recipes.paging_scenario(), golden["trace"]):
        kind, sid = op[0], op[1]
        if kind == "ensure":
            tables.ensure_capacity(sid, op[2])
        elif kind == "advance":
            tables.advance(sid, op[2])
        else:
            tables.release(sid)
        assert {s: t for s, t in sorted(tables.tables.items())} == expected["tables"]
        assert {s: n for s, n in sorted(tables.lengths.items())} == expected["lengths"]
        assert len(tables.alloc.free) == expected["free"]
    step = golden["step"]
    meta = ragged_metadata([tables.tables[s] for s in step["ids"]], step["contexts"], step["qlens"], 16)
    assert meta["slot_mapping"] == step["slots"]


@pytest.mark.parametrize("name", recipes.DECODE_CASES)
def test_decode_oracle_matches_reference(name):
    case = recipes.decode_case(name)
    golden = torch.load(GOLDEN / f"decode_{name}.pt")["out"]
    out = oatt.paged_decode(case["query"], case["key_cache"], case["value_cache"], case["tables"],
                            case["seq_lens"], case["layer"])
    assert out.dtype == golden.dtype
    if golden.dtype == torch.bfloat16:
        torch.testing.assert_close(out.float(), golden.float(), atol=8e-3, rtol=0)
    else:
        torch.testing.assert_close(out, golden, atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("name", recipes.RAGGED_CASES)
def test_ragged_oracle_matches_reference(name):
    c = recipes.ragged_case(name)
    golden = torch.load(GOLDEN / f"ragged_{name}.pt")
    cache = OracleCache(c["num_blocks"], c["block_size"], 1, c["hkv"], 64, c["dtype"])
    for sid, n in c["warmup"]:
        cache.tables.ensure_capacity(sid, n)
    for sid in c["release"]:
        cache.tables.release(sid)
    for sid, ctx, (hk, hv), ql in zip(c["ids"], c["contexts"], c["history"], c["qlens"]):
        cache.tables.ensure_capacity(sid, ctx + ql)
        if ctx:
            cache.write(0, sid, 0, hk, hv)
            cache.tables.advance(sid, ctx)
    for sid in c["ids"]:
        assert cache.tables.tables[sid] == golden["tables"][sid]
    w = c["weights"]
    x = c["x"]
    T = x.shape[0]
    q = (x @ w["q_proj.weight"].t()).view(T, c["hq"], 64)
    k = (x @ w["k_proj.weight"].t()).view(T, c["hkv"], 64)
    v = (x @ w["v_proj.weight"].t()).view(T, c["hkv"], 64)
    positions = torch.cat([torch.arange(ctx, ctx + q_) for ctx, q_ in zip(c["contexts"], c["qlens"])])
    f = inv_freq(64, c["rope_theta"])
    q, k = rope(q, positions, f), rope(k, positions, f)
    start = 0
    for sid, ctx, ql in zip(c["ids"], c["contexts"], c["qlens"]):
        cache.write(0, sid, ctx, k[start : start + ql], v[start : start + ql])
        start += ql
    tables = [cache.tables.tables[s] for s in c["ids"]]
    attn = oatt.varlen_attention(q, cache.keys, cache.values, tables, c["contexts"], c["qlens"], 0)
    out = attn.reshape(T, -1) @ w["o_proj.weight"].t()
    for sid, ctx, ql in zip(c["ids"], c["contexts"], c["qlens"]):
        gk = oatt.gather_sequence(cache.keys, 0, cache.tables.tables[sid], ctx + ql)
        gv = oatt.gather_sequence(cache.values, 0, cache.tables.tables[sid], ctx + ql)
        assert torch.equal(gk, golden["keys"][sid]) and torch.equal(gv, golden["values"][sid])
    tol = dict(atol=2e-2, rtol=0) if c["dtype"] == torch.bfloat16 else dict(atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(out.float(), golden["out"].float(), **tol)
