"""Host-side paging state is bit-identical to the reference (allocator, block tables,
sequence lengths, device-table mirror), checked on CPU caches (no kernels)."""

import json
import random
from pathlib import Path

import pytest
import torch

import recipes
from nano_infer_engine_b200.block_allocator import BlockAllocator
from nano_infer_engine_b200.paged_cache import PagedKVCache
from oracle.paging import OracleTables

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cache(num_blocks=4, block_size=4, **kw):
    args = dict(num_blocks=num_blocks, block_size=block_size, num_layers=2, kv_head_num=2, head_dim=4,
                dtype=torch.float32, device="cpu")
    args.update(kw)
    return PagedKVCache(**args)


# ------------------------------------------------------------ allocator
def test_allocator_order_and_reuse():
    a = BlockAllocator(4)
    assert a.allocate(2) == [0, 1]
    assert (a.free_block_count, a.allocated_block_count) == (2, 2)
    b = BlockAllocator(4)
    got = b.allocate(4)
    b.free([got[1], got[3]])
    assert b.allocate(2) == [got[1], got[3]]


def test_allocator_errors_are_atomic():
    a = BlockAllocator(3)
    with pytest.raises(ValueError, match="not enough free blocks"):
        a.allocate(4)
    assert a.free_block_count == 3
    bid = a.allocate()[0]
    with pytest.raises(ValueError, match="same block more than once"):
        a.free([bid, bid])
    with pytest.raises(ValueError, match="block is not allocated"):
        a.free([bid, 1])
    assert (a.free_block_count, a.allocated_block_count) == (2, 1)
    with pytest.raises(ValueError, match="block ID out of range"):
        a.free([7])
    with pytest.raises(TypeError, match="block IDs must be integers"):
        a.free([True])
    for bad in (0, -1):
        with pytest.raises(ValueError, match="num_blocks must be positive"):
            BlockAllocator(bad)
        with pytest.raises(ValueError, match="block_count must be positive"):
            a.allocate(bad)
    for bad in (True, 1.5):
        with pytest.raises(TypeError, match="num_blocks must be an integer"):
            BlockAllocator(bad)
        with pytest.raises(TypeError, match="block_count must be an integer"):
            a.allocate(bad)


# ----------------------------------------------------------- block tables
def test_paging_trace_matches_reference_golden():
    golden = json.loads((GOLDEN / "paging.json").read_text())
    cache = PagedKVCache(32, 16, 1, 1, 16, torch.float32, "cpu")
    for op, want in zip(recipes.paging_scenario(), golden["trace"]):
        kind, sid = op[0], op[1]
        if kind == "ensure":
            cache.ensure_capacity(sid, op[2])
        elif kind == "advance":
            cache.advance(sid, op[2])
        else:
            cache.release(sid)
        assert {s: list(cache.get_block_table(s)) for s in sorted(cache._block_tables)} == want["tables"]
        assert {s: cache.get_sequence_length(s) for s in sorted(cache._block_tables)} == want["lengths"]
        assert cache.allocator.free_block_count == want["free"]
        _check_mirror(cache)


def _check_mirror(cache: PagedKVCache) -> None:
    """The host copy of the device block-table array holds exactly the live tables."""
    for sid, table in cache._block_tables.items():
        row = cache._table_host[cache.table_row(sid)].tolist()
        assert row[: len(table)] == table
        assert all(v == -1 for v in row[len(table):])
    live_rows = {cache.table_row(s) for s in cache._block_tables}
    assert len(live_rows) == len(cache._block_tables)


@pytest.mark.parametrize("seed", range(5))
def test_random_differential_against_oracle(seed):
    rng = random.Random(seed)
    nb, bs = 64, 16
    cache = PagedKVCache(nb, bs, 1, 1, 16, torch.float32, "cpu")
    ref = OracleTables(nb, bs)
    names = [f"s{i}" for i in range(12)]
    for _ in range(400):
        sid = rng.choice(names)
        op = rng.random()
        if op < 0.55:
            n = rng.randint(1, 200)
            try:
                ref.ensure_capacity(sid, n)
                ok = True
            except ValueError:
                ok = False
            if ok:
                cache.ensure_capacity(sid, n)
            else:
                with pytest.raises(ValueError, match="not enough free blocks"):
                    cache.ensure_capacity(sid, n)
        elif op < 0.8 and sid in ref.tables:
            cap = len(ref.tables[sid]) * bs - ref.lengths[sid]
            if cap > 0:
                k = rng.randint(1, cap)
                ref.advance(sid, k)
                cache.advance(sid, k)
        elif sid in ref.tables:
            ref.release(sid)
            cache.release(sid)
        assert {s: list(t) for s, t in cache._block_tables.items()} == ref.tables
        assert cache._sequence_lengths == ref.lengths
        assert cache.allocator.free_block_count == len(ref.alloc.free)
        _check_mirror(cache)


def test_cache_validation_messages():
    c = _cache()
    with pytest.raises(ValueError, match="required_tokens must be positive"):
        c.ensure_capacity("a", 0)
    with pytest.raises(TypeError, match="required_tokens must be an integer"):
        c.ensure_capacity("a", 1.5)
    with pytest.raises(TypeError, match="sequence_id must be a string"):
        c.get_block_table(None)
    with pytest.raises(ValueError, match="sequence_id must not be empty"):
        c.get_block_table("")
    with pytest.raises(KeyError, match="request-a"):
        c.get_block_table("request-a")
    c.ensure_capacity("a", 4)
    c.advance("a", 4)
    with pytest.raises(IndexError, match="exceeds allocated capacity"):
        c.advance("a", 1)
    assert c.get_sequence_length("a") == 4
    with pytest.raises(ValueError, match="not enough free blocks"):
        c.ensure_capacity("b", 17)
    with pytest.raises(KeyError):
        c.get_block_table("b")


def test_release_keeps_table_when_free_fails(monkeypatch):
    c = _cache(num_blocks=2)
    c.ensure_capacity("a", 4)
    table = c.get_block_table("a")

    def boom(ids):
        raise RuntimeError("simulated allocator failure")

    monkeypatch.setattr(c.allocator, "free", boom)
    with pytest.raises(RuntimeError, match="simulated allocator failure"):
        c.release("a")
    assert c.get_block_table("a") == table
    _check_mirror(c)


def test_mirror_grows_rows_and_columns():
    c = PagedKVCache(4096, 1, 1, 1, 4, torch.float32, "cpu")
    for i in range(40):
        c.ensure_capacity(f"s{i}", 1 + i * 3)
    c.ensure_capacity("s3", 500)
    _check_mirror(c)
    for i in range(0, 40, 3):
        c.release(f"s{i}")
    c.ensure_capacity("new", 9)
    _check_mirror(c)


def test_cpu_cache_data_ops_fail_loudly():
    c = _cache()
    c.ensure_capacity("a", 2)
    with pytest.raises(RuntimeError, match="require a CUDA cache|require CUDA tensors"):
        c.write(0, "a", 0, torch.zeros(2, 2, 4), torch.zeros(2, 2, 4))


def test_layer_loop_eligibility_follows_the_python_loop_checks():
    """The C++ layer loop runs only when the Python loop's fused-weight, hook and bias checks hold."""
    from torch import nn

    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    cfg = LlamaConfig(vocab_size=64, hidden_size=128, mlp_inner_size=256, num_layers=2, q_head_num=2,
                      kv_head_num=1, max_seq_len=256)
    model = build_random_llama(cfg, 3, 0.02, torch.bfloat16, "cpu")
    model._ensure_fused()
    args = model._layer_loop_args(torch.bfloat16)
    assert args is not None
    weights, eps = args
    assert len(weights) == 6 * cfg.num_layers and len(eps) == 2 * cfg.num_layers
    assert model._layer_loop_args(torch.float32) is None  # dtype mismatch
    o_proj = model.decoders[1].attn.o_proj
    handle = o_proj.register_forward_hook(lambda *a: None)
    assert model._layer_loop_args(torch.bfloat16) is None
    handle.remove()
    assert model._layer_loop_args(torch.bfloat16) is not None
    down = model.decoders[0].ffn.down_proj
    down.bias = nn.Parameter(torch.zeros(down.out_features, dtype=torch.bfloat16))
    assert model._layer_loop_args(torch.bfloat16) is None
    down.bias = None
    attn = model.decoders[0].attn
    attn.k_proj.weight = nn.Parameter(attn.k_proj.weight.detach().clone())  # no longer a view of the fused buffer
    assert model._layer_loop_args(torch.bfloat16) is None


def test_reserve_table_grows_once_and_never_shrinks():
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    cache = PagedKVCache(64, 16, 1, 1, 4, torch.float32, "cpu")
    rows, cols = cache._table_host.shape
    cache.reserve_table(rows * 4, cols * 2)
    assert cache._table_host.shape == (rows * 4, cols * 2)
    cache.reserve_table(1, 1)  # smaller: nothing changes
    assert cache._table_host.shape == (rows * 4, cols * 2)
    # sequences keep their tables across a reservation
    cache.ensure_capacity("a", 40)
    before = cache.get_block_table("a")
    cache.reserve_table(rows * 8, cols * 2)
    assert cache.get_block_table("a") == before
    assert cache._table_host[cache.table_row("a"), : len(before)].tolist() == list(before)
