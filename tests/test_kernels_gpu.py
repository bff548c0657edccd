"""Kernel parity on the GPU: every C-ABI kernel against the CPU oracle / reference goldens.

Integer and byte work (packing, slot write, gather, block copy) must be
bit-exact; attention must be within max-abs 2e-2 (bf16) / 1e-4 (fp32) of the
oracle.
"""

from pathlib import Path

import pytest
import torch

import recipes
from oracle import attention as oatt
from oracle.paging import OracleTables, ragged_metadata

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def ops():
    from nano_infer_engine_b200 import ops as _ops

    return _ops


def _tables_tensor(tables, device, width=None):
    width = width or max(len(t) for t in tables)
    out = torch.full((len(tables), width), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        out[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
    return out.to(device)


def _random_layout(num_blocks, seq_lens, bs, seed):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, at = [], 0
    for n in seq_lens:
        nb = (n + bs - 1) // bs
        tables.append(perm[at : at + nb])
        at += nb
    return tables


# ------------------------------------------------------------------ (a)
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_pack_ragged_bit_exact(cuda, seed):
    g = torch.Generator().manual_seed(seed)
    bs, nb = 16, 4096
    R = int(torch.randint(1, 300, (1,), generator=g))
    contexts = torch.randint(0, 3000, (R,), generator=g).tolist()
    qlens = [1 if torch.rand(1, generator=g).item() < 0.6 else int(torch.randint(2, 200, (1,), generator=g)) for _ in range(R)]
    tables = _random_layout(nb * 8, [c + q for c, q in zip(contexts, qlens)], bs, seed)
    tables = [[b % nb for b in t] for t in tables]
    rows = torch.randperm(R, generator=g).tolist()  # requests live in arbitrary table rows
    table_dev = torch.full((R, max(len(t) for t in tables) + 3), -1, dtype=torch.int32)
    for r, t in zip(rows, tables):
        table_dev[r, : len(t)] = torch.tensor(t, dtype=torch.int32)
    plan = torch.tensor([rows, contexts, qlens], dtype=torch.int32).to(cuda)
    meta = ops().pack_ragged(plan, sum(qlens), table_dev.to(cuda), bs, nb,
                             num_decode=sum(q == 1 for q in qlens), max_query_len=max(qlens))
    want = ragged_metadata(tables, contexts, qlens, bs)
    assert meta.query_start_loc.cpu().tolist() == want["query_start_loc"]
    assert meta.positions.cpu().tolist() == want["positions"]
    assert meta.slot_mapping.cpu().tolist() == want["slot_mapping"]
    assert meta.seq_lens.cpu().tolist() == want["seq_lens"]
    assert meta.last_token_index.cpu().tolist() == want["last_token_index"]
    counts = meta.list_counts.cpu().tolist()
    assert meta.decode_list[: counts[0]].cpu().tolist() == want["decode_list"]
    assert meta.prefill_list[: counts[1]].cpu().tolist() == want["prefill_list"]
    tok_req = meta.token_request.cpu().tolist()
    assert tok_req == [r for r, q in enumerate(qlens) for _ in range(q)]
    ops().check_device_errors(cuda)


def test_pack_flags_unallocated_positions(cuda):
    table = torch.tensor([[3, -1]], dtype=torch.int32, device=cuda)
    plan = torch.tensor([[0], [10], [10]], dtype=torch.int32, device=cuda)  # positions 10..19, block 1 missing
    meta = ops().pack_ragged(plan, 10, table, 16, 8, num_decode=0, max_query_len=10)
    slots = meta.slot_mapping.cpu().tolist()
    assert slots[:6] == [3 * 16 + p for p in range(10, 16)]
    assert slots[6:] == [-1] * 4
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        ops().check_device_errors(cuda)


# ------------------------------------------------------------------ (b)
@pytest.mark.parametrize("dtype,hkv,hd", [(torch.bfloat16, 8, 64), (torch.float32, 2, 64), (torch.bfloat16, 2, 3)])
def test_write_kv_bit_exact(cuda, dtype, hkv, hd):
    g = torch.Generator().manual_seed(5)
    L, nb, bs, T = 3, 64, 16, 200
    kc = torch.randn(L, nb, bs, hkv, hd, generator=g).to(dtype)
    vc = torch.randn(L, nb, bs, hkv, hd, generator=g).to(dtype)
    k = torch.randn(T, hkv, hd, generator=g).to(dtype)
    v = torch.randn(T, hkv, hd, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:T]
    slots[7] = -1  # skipped, like a slot the packer could not resolve
    want_k, want_v = kc.clone(), vc.clone()
    for t, s in enumerate(slots.tolist()):
        if s >= 0:
            want_k[1, s // bs, s % bs] = k[t]
            want_v[1, s // bs, s % bs] = v[t]
    dk, dv = kc.to(cuda), vc.to(cuda)
    ops().write_kv(k.to(cuda), v.to(cuda), dk, dv, 1, slots.to(cuda))
    assert torch.equal(dk.cpu(), want_k) and torch.equal(dv.cpu(), want_v)
    ops().check_device_errors(cuda)


def test_gather_kv_bit_exact(cuda):
    g = torch.Generator().manual_seed(6)
    kc = torch.randn(2, 40, 16, 8, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(2, 40, 16, 8, 64, generator=g).to(torch.bfloat16)
    table = [7, 3, 30, 11]
    n = 53
    gk, gv = ops().gather_kv(kc.to(cuda), vc.to(cuda), 1, torch.tensor(table, dtype=torch.int32, device=cuda), n)
    assert torch.equal(gk.cpu(), oatt.gather_sequence(kc, 1, table, n))
    assert torch.equal(gv.cpu(), oatt.gather_sequence(vc, 1, table, n))


# ------------------------------------------------------------------ (e)
@pytest.mark.parametrize("length", [16, 37, 1])
def test_copy_blocks_export_semantics(cuda, length):
    """Block copy with a zeroed tail == reference export_sequence (paged_cache.py:145-180)."""
    g = torch.Generator().manual_seed(length)
    L, nb, bs = 3, 20, 16
    kc = torch.randn(L, nb, bs, 8, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(L, nb, bs, 8, 64, generator=g).to(torch.bfloat16)
    n = (length + bs - 1) // bs
    src = torch.randperm(nb, generator=g)[:n].tolist()
    dst_pool_k = torch.full((L, nb, bs, 8, 64), 7.0, dtype=torch.bfloat16)
    dst_pool_v = dst_pool_k.clone()
    dst = torch.randperm(nb, generator=g)[:n].tolist()
    dk, dv = dst_pool_k.to(cuda), dst_pool_v.to(cuda)
    ops().copy_blocks(kc.to(cuda), vc.to(cuda), torch.tensor(src, dtype=torch.int32, device=cuda), dk, dv,
                      torch.tensor(dst, dtype=torch.int32, device=cuda), n, length % bs)
    want_k, want_v = dst_pool_k.clone(), dst_pool_v.clone()
    for j, (s, d) in enumerate(zip(src, dst)):
        want_k[:, d] = kc[:, s]
        want_v[:, d] = vc[:, s]
    tail = length % bs
    if tail:
        want_k[:, dst[-1], tail:] = 0
        want_v[:, dst[-1], tail:] = 0
    assert torch.equal(dk.cpu(), want_k) and torch.equal(dv.cpu(), want_v)


# ------------------------------------------------------------------ (c)
@pytest.mark.parametrize("name", recipes.DECODE_CASES)
def test_decode_matches_reference_golden(cuda, name):
    case = recipes.decode_case(name)
    golden = torch.load(GOLDEN / f"decode_{name}.pt")["out"]
    tables = _tables_tensor(case["tables"], cuda)
    lens = torch.tensor(case["seq_lens"], dtype=torch.int32, device=cuda)
    out = ops().paged_decode(case["query"].to(cuda), case["key_cache"].to(cuda), case["value_cache"].to(cuda),
                             case["layer"], tables, lens)
    ops().check_device_errors(cuda)
    tol = TOL[golden.dtype]
    torch.testing.assert_close(out.cpu().float(), golden.float(), atol=tol, rtol=0)


@pytest.mark.parametrize("seed,B,max_ctx,hkv", [(0, 64, 3000, 8), (1, 7, 20000, 8), (2, 130, 600, 8),
                                                (3, 1, 29600, 8), (4, 20, 2500, 16)])
def test_fast_decode_against_oracle(cuda, seed, B, max_ctx, hkv):
    """bf16 / hd 64 / bs 16 split-K kernel, ragged lengths incl. 1 and block-aligned.

    16 kv heads is the widest group layout the kernel takes (one warp per kv
    head, a shallower pipeline so the CTA's tiles fit in shared memory)."""
    g = torch.Generator().manual_seed(seed)
    bs = 16
    lens = torch.randint(1, max_ctx + 1, (B,), generator=g).tolist()
    lens[0] = 1
    if B > 2:
        lens[1] = 16 * 7
    total_blocks = sum((n + bs - 1) // bs for n in lens)
    nb = total_blocks + 37
    tables = _random_layout(nb, lens, bs, seed)
    kc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    q = torch.randn(B, 32, 64, generator=g).to(torch.bfloat16)
    dk, dv = kc.to(cuda), vc.to(cuda)
    # poison the unused tail rows: masked positions must not leak (NaN * 0)
    for t, n in zip(tables, lens):
        if n % bs:
            dk[0, t[-1], n % bs :] = float("nan")
            dv[0, t[-1], n % bs :] = float("nan")
    out = ops().paged_decode(q.to(cuda), dk, dv, 0, _tables_tensor(tables, cuda),
                             torch.tensor(lens, dtype=torch.int32, device=cuda))
    ops().check_device_errors(cuda)
    want = oatt.paged_decode(q, kc, vc, tables, lens, 0)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.cpu().float(), want.float(), atol=2e-2, rtol=0)


def test_decode_with_indirection(cuda):
    """req_list / table_rows / q_rows indirection as used for the decode rows of a mixed step."""
    g = torch.Generator().manual_seed(9)
    lens = [50, 1, 333, 17]
    tables = _random_layout(80, lens, 16, 9)
    kc = torch.randn(1, 80, 16, 8, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(1, 80, 16, 8, 64, generator=g).to(torch.bfloat16)
    q = torch.randn(10, 32, 64, generator=g).to(torch.bfloat16)
    # requests 0..3 live in table rows 2,0,3,1; their query rows are 9,4,0,6; decode only 1 and 2
    rows = [2, 0, 3, 1]
    qrows = [9, 4, 0, 6]
    t = [None] * 4
    for r, row in enumerate(rows):
        t[row] = tables[r]
    out = torch.zeros(10, 32, 64, dtype=torch.bfloat16, device=cuda)
    ops().paged_decode(q.to(cuda), kc.to(cuda), vc.to(cuda), 0, _tables_tensor(t, cuda),
                       torch.tensor(lens, dtype=torch.int32, device=cuda), out=out,
                       table_rows=torch.tensor(rows, dtype=torch.int32, device=cuda),
                       q_rows=torch.tensor(qrows, dtype=torch.int64, device=cuda),
                       req_list=torch.tensor([1, 2], dtype=torch.int32, device=cuda), num_requests=2)
    want = oatt.paged_decode(q[[4, 0]], kc, vc, [tables[1], tables[2]], [lens[1], lens[2]], 0)
    got = out.cpu()
    torch.testing.assert_close(got[[4, 0]].float(), want.float(), atol=2e-2, rtol=0)
    untouched = [i for i in range(10) if i not in (4, 0)]
    assert torch.count_nonzero(got[untouched]) == 0


def test_decode_bad_block_id_sets_flag_without_fault(cuda):
    kc = torch.zeros(1, 8, 16, 8, 64, dtype=torch.bfloat16, device=cuda)
    q = torch.zeros(1, 32, 64, dtype=torch.bfloat16, device=cuda)
    table = torch.tensor([[1, 99]], dtype=torch.int32, device=cuda)
    ops().paged_decode(q, kc, kc, 0, table, torch.tensor([20], dtype=torch.int32, device=cuda))
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        ops().check_device_errors(cuda)
    torch.cuda.synchronize()


# ------------------------------------------------------------------ (d)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_varlen_against_oracle(cuda, dtype):
    g = torch.Generator().manual_seed(21)
    contexts = [0, 7, 300, 1000, 16, 5]
    qlens = [5, 16, 129, 64, 1, 2]
    bs, hkv, hq = 16, 8, 32
    lens = [c + q for c, q in zip(contexts, qlens)]
    nb = sum((n + bs - 1) // bs for n in lens) + 11
    tables = _random_layout(nb, lens, bs, 21)
    kc = torch.randn(2, nb, bs, hkv, 64, generator=g).to(dtype)
    vc = torch.randn(2, nb, bs, hkv, 64, generator=g).to(dtype)
    q = torch.randn(sum(qlens), hq, 64, generator=g).to(dtype)
    qsl = [0]
    for n in qlens:
        qsl.append(qsl[-1] + n)
    out = ops().varlen_attention(q.to(cuda), kc.to(cuda), vc.to(cuda), 1, _tables_tensor(tables, cuda),
                                 torch.tensor(lens, dtype=torch.int32, device=cuda),
                                 torch.tensor(qsl, dtype=torch.int64, device=cuda), max(qlens))
    ops().check_device_errors(cuda)
    want = oatt.varlen_attention(q, kc, vc, tables, contexts, qlens, 1)
    torch.testing.assert_close(out.cpu().float(), want.float(), atol=TOL[dtype], rtol=0)


@pytest.mark.parametrize("seed,contexts,qlens", [
    (30, [0, 0, 5], [1, 2, 17]),
    (31, [0, 130, 4000, 8100, 37], [128, 128, 128, 128, 300]),
    (32, [0], [1000]),
    (33, [15, 16, 17, 255, 256, 257], [2, 16, 127, 129, 3, 64]),
    (34, [1000, 3000, 16, 0], [128, 50, 1, 200]),
])
@pytest.mark.parametrize("split", [False, True])
def test_tensor_core_varlen_against_oracle(cuda, seed, contexts, qlens, split):
    """tcgen05 path (bf16, hd 64, bs 16): multi-tile queries, long contexts, ragged
    ends; stale rows past each sequence end hold NaN and must not leak.  With
    ``split`` (a workspace) the persistent grid cuts segments across CTAs and
    merges their partials inside the kernel; without it each CTA takes one
    whole segment."""
    g = torch.Generator().manual_seed(seed)
    bs, hkv, hq = 16, 8, 32
    lens = [c + q for c, q in zip(contexts, qlens)]
    nb = sum((n + bs - 1) // bs for n in lens) + 5
    tables = _random_layout(nb, lens, bs, seed)
    kc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    q = torch.randn(sum(qlens), hq, 64, generator=g).to(torch.bfloat16)
    dk, dv = kc.to(cuda), vc.to(cuda)
    for t, n in zip(tables, lens):
        if n % bs:
            dk[0, t[-1], n % bs:] = float("nan")
            dv[0, t[-1], n % bs:] = float("nan")
    qsl = [0]
    for n in qlens:
        qsl.append(qsl[-1] + n)
    out = ops().varlen_attention(q.to(cuda), dk, dv, 0, _tables_tensor(tables, cuda),
                                 torch.tensor(lens, dtype=torch.int32, device=cuda),
                                 torch.tensor(qsl, dtype=torch.int64, device=cuda), max(qlens),
                                 max_seq_len=max(lens) if split else None)
    ops().check_device_errors(cuda)
    want = oatt.varlen_attention(q, kc, vc, tables, contexts, qlens, 0)
    got = out.cpu().float()
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want.float(), atol=2e-2, rtol=0)


def test_mixed_step_config4_shape(cuda):
    """BASELINE config 4 at reduced context: 8 prefill chunks of 128 + 120 decode rows,
    prefill first, through pack -> write -> decode + varlen, against the oracle."""
    g = torch.Generator().manual_seed(40)
    bs, hkv, hq = 16, 8, 32
    pf_ctx = torch.randint(0, 2048, (8,), generator=g).tolist()
    dec_ctx = torch.randint(256, 4096, (120,), generator=g).tolist()
    contexts = pf_ctx + dec_ctx
    qlens = [128] * 8 + [1] * 120
    lens = [c + q for c, q in zip(contexts, qlens)]
    nb = sum((n + bs - 1) // bs for n in lens) + 3
    tables = _random_layout(nb, lens, bs, 40)
    kc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    vc = torch.randn(1, nb, bs, hkv, 64, generator=g).to(torch.bfloat16)
    T = sum(qlens)
    q = torch.randn(T, hq, 64, generator=g).to(torch.bfloat16)
    k_new = torch.randn(T, hkv, 64, generator=g).to(torch.bfloat16)
    v_new = torch.randn(T, hkv, 64, generator=g).to(torch.bfloat16)
    R = len(qlens)
    plan = torch.tensor([list(range(R)), contexts, qlens], dtype=torch.int32).to(cuda)
    meta = ops().pack_ragged(plan, T, _tables_tensor(tables, cuda), bs, nb, num_decode=120, max_query_len=128)
    dk, dv = kc.to(cuda), vc.to(cuda)
    qd = q.to(cuda)
    ops().write_kv(k_new.to(cuda), v_new.to(cuda), dk, dv, 0, meta.slot_mapping)
    out = torch.empty_like(qd)
    ops().paged_decode(qd, dk, dv, 0, meta.block_tables, meta.seq_lens, out=out, table_rows=meta.table_rows,
                       q_rows=meta.query_start_loc, req_list=meta.decode_list, num_requests=meta.num_decode)
    ops().varlen_attention(qd, dk, dv, 0, meta.block_tables, meta.seq_lens, meta.query_start_loc, 128, out=out,
                           table_rows=meta.table_rows, req_list=meta.prefill_list, num_requests=meta.num_prefill)
    ops().check_device_errors(cuda)
    # oracle: write the new rows on the CPU copy, then attend
    kc2, vc2 = kc.clone(), vc.clone()
    pos = 0
    for t, c, ql in zip(tables, contexts, qlens):
        for j in range(ql):
            p = c + j
            kc2[0, t[p // bs], p % bs] = k_new[pos]
            vc2[0, t[p // bs], p % bs] = v_new[pos]
            pos += 1
    assert torch.equal(dk.cpu(), kc2) and torch.equal(dv.cpu(), vc2)
    want = oatt.varlen_attention(q, kc2, vc2, tables, contexts, qlens, 0)
    torch.testing.assert_close(out.cpu().float(), want.float(), atol=2e-2, rtol=0)


# ------------------------------------------------ fused elementwise stages
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_rope_write_matches_torch_ops(cuda, dtype):
    """RoPE + slot write equals the torch op chain (reference layers/rope.py:6-23) bit for bit."""
    from nano_infer_engine_b200.layers.rope import RopeScale, apply_rotary

    g = torch.Generator().manual_seed(50)
    T, hq, hkv, d, bs, nb = 37, 32, 8, 64, 16, 40
    q = torch.randn(T, hq * d, generator=g).to(dtype).to(cuda)
    k = torch.randn(T, hkv * d, generator=g).to(dtype).to(cuda)
    v = torch.randn(T, hkv * d, generator=g).to(dtype).to(cuda)
    pos = torch.randint(0, 30000, (T,), generator=g).to(cuda)
    sin, cos = RopeScale(d).sin_cos(pos, dtype)
    kc = torch.zeros(2, nb, bs, hkv, d, dtype=dtype, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, generator=g)[:T].to(cuda)
    qr = ops().rope_write_kv(q, k, v, sin, cos, kc, vc, 1, slots, hq)
    want_q = apply_rotary(q.view(T, hq, d), sin, cos)
    want_k = apply_rotary(k.view(T, hkv, d), sin, cos)
    assert torch.equal(qr, want_q)
    flat_k = kc[1].view(-1, hkv, d)
    flat_v = vc[1].view(-1, hkv, d)
    assert torch.equal(flat_k[slots], want_k)
    assert torch.equal(flat_v[slots], v.view(T, hkv, d))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_silu_mul_and_add_rmsnorm_match_torch_ops(cuda, dtype):
    from nano_infer_engine_b200.layers.rms_norm import RmsNorm

    g = torch.Generator().manual_seed(51)
    gate = torch.randn(19, 8192, generator=g).to(dtype).to(cuda)
    up = torch.randn(19, 8192, generator=g).to(dtype).to(cuda)
    assert torch.equal(ops().silu_mul(gate, up), torch.nn.functional.silu(gate) * up)
    x = torch.randn(19, 2048, generator=g).to(dtype).to(cuda)
    r = torch.randn(19, 2048, generator=g).to(dtype).to(cuda)
    norm = RmsNorm(2048, 1e-5).to(cuda)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(2048, generator=g) + 0.5)
    norm = norm.to(dtype)
    total, out = ops().add_rmsnorm(x, r, norm.weight, 1e-5)
    assert torch.equal(total, x + r)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    torch.testing.assert_close(out.float(), norm(x + r).float(), atol=tol, rtol=tol)
    _, plain = ops().add_rmsnorm(x, None, norm.weight, 1e-5)
    torch.testing.assert_close(plain.float(), norm(x).float(), atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_kernels_unaligned_fallbacks_match_torch(cuda, dtype):
    """Shapes and views that are not 16-byte aligned take the scalar kernels: same results."""
    from nano_infer_engine_b200.layers.rms_norm import RmsNorm
    from nano_infer_engine_b200.layers.rope import RopeScale, apply_rotary

    g = torch.Generator().manual_seed(52)
    gate = torch.randn(5, 8190, generator=g).to(dtype).to(cuda)
    up = torch.randn(5, 8190, generator=g).to(dtype).to(cuda)
    assert torch.equal(ops().silu_mul(gate, up), torch.nn.functional.silu(gate) * up)
    x = torch.randn(5, 2046, generator=g).to(dtype).to(cuda)
    norm = RmsNorm(2046, 1e-5).to(cuda).to(dtype)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    _, out = ops().add_rmsnorm(x, None, norm.weight, 1e-5)
    torch.testing.assert_close(out.float(), norm(x).float(), atol=tol, rtol=tol)
    T, hq, hkv, d = 9, 4, 2, 64
    base = torch.randn(T, hq * d + 1, generator=g).to(dtype).to(cuda)
    q = base[:, 1:]  # 2- or 4-byte offset: scalar path
    k = torch.randn(T, hkv * d, generator=g).to(dtype).to(cuda)
    v = torch.randn(T, hkv * d, generator=g).to(dtype).to(cuda)
    sin, cos = RopeScale(d).sin_cos(torch.arange(T, device=cuda) * 7, dtype)
    kc = torch.zeros(1, 4, 16, hkv, d, dtype=dtype, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.arange(T, device=cuda) * 3
    qr = ops().rope_write_kv(q, k, v, sin, cos, kc, vc, 0, slots, hq)
    assert torch.equal(qr, apply_rotary(q.reshape(T, hq, d), sin, cos))
    assert torch.equal(kc[0].view(-1, hkv, d)[slots], apply_rotary(k.view(T, hkv, d), sin, cos))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_embed_rows_bit_exact_and_bad_id_flag(cuda, dtype):
    g = torch.Generator().manual_seed(53)
    table = torch.randn(1000, 256, generator=g).to(dtype).to(cuda)
    ids = torch.randint(0, 1000, (37,), generator=g).to(cuda)
    assert torch.equal(ops().embed_rows(ids, table), torch.nn.functional.embedding(ids, table))
    bad = torch.tensor([3, 1000, -1, 7], device=cuda)
    out = ops().embed_rows(bad, table)
    assert torch.equal(out[0], table[3]) and torch.equal(out[3], table[7])
    assert not out[1].any() and not out[2].any()
    with pytest.raises(RuntimeError, match="token id outside the vocabulary"):
        ops().check_device_errors(cuda)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(1, 7), (16, 128256), (64, 1024), (3, 100003)])
def test_argmax_rows_matches_torch(cuda, dtype, rows, cols):
    g = torch.Generator().manual_seed(rows * 31 + cols)
    x = torch.randn(rows, cols, generator=g).to(dtype)
    # exact ties (first index wins) and a NaN row (first NaN wins)
    x[0, cols // 3] = 50.0
    x[0, cols // 2] = 50.0
    if rows > 2:
        x[2, cols - 1] = float("nan")
        x[2, 1] = float("nan")
    x = x.to(cuda)
    for _ in range(3):  # counters must be reset by every call
        got = ops().argmax_rows(x)
        assert torch.equal(got, x.argmax(dim=-1))
    view = x[:, : cols - 1] if cols > 1 else x  # row stride larger than the row
    assert torch.equal(ops().argmax_rows(view), view.argmax(dim=-1))


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (5, 3072, 2048), (16, 2048, 8192), (16, 16384, 2048),
                                   (7, 640, 640), (16, 128, 8192)])
def test_stream_linear_matches_fp32_reference(cuda, m, n, k):
    """nie_linear (weight streaming, K split over a cluster, partials merged in shared memory) against torch fp32.

    Tolerance: fp32 accumulation in a different order, then one bf16 rounding of
    the output, so |err| <= 1 bf16 ulp of |y| plus fp32 noise: atol 1e-3 on
    outputs of scale ~0.5, rtol 2^-7."""
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16).to(cuda)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).to(cuda)
    before = ops().LAUNCHES
    y = ops().linear_stream(x, w)
    assert ops().LAUNCHES == before + 1
    ops().check_device_errors(cuda)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y.float(), ref, atol=1e-3, rtol=2 ** -7)
    # same bits on a second call (fixed merge order), also after a call of another shape
    ops().linear_stream(x[:, :64].contiguous(), w[:128, :64].contiguous())
    assert torch.equal(ops().linear_stream(x, w), y)
    ops().check_device_errors(cuda)


def test_stream_linear_strided_rows_and_routing(cuda):
    """x rows with a stride (a column slice) use the kernel; ops.linear routes K >= N
    matrices to it and everything else (more rows, K < N, ragged N) to torch."""
    g = torch.Generator().manual_seed(1)
    big = torch.randn(9, 3072, generator=g).to(torch.bfloat16).to(cuda)
    x = big[:, 1024:3072]
    w = (torch.randn(256, 2048, generator=g) / 45).to(torch.bfloat16).to(cuda)
    assert ops().linear_eligible(x, w)
    torch.testing.assert_close(ops().linear(x, w).float(), x.float() @ w.float().T, atol=1e-3, rtol=2 ** -7)
    before = ops().LAUNCHES
    ops().linear(x, w)
    assert ops().LAUNCHES == before + 1
    x17 = torch.randn(17, 2048, generator=g).to(torch.bfloat16).to(cuda)
    assert not ops().linear_eligible(x17, w)
    assert torch.equal(ops().linear(x17, w), torch.nn.functional.linear(x17, w))
    wide = torch.randn(4096, 2048, generator=g).to(torch.bfloat16).to(cuda)
    assert not ops().linear_eligible(x, wide)
    w100 = torch.randn(100, 2048, generator=g).to(torch.bfloat16).to(cuda)
    assert not ops().linear_eligible(x, w100)
    ops().check_device_errors(cuda)


def test_overlapped_decode_sees_the_rope_kernel_writes(cuda):
    """nie_paged_decode_overlapped right after the RoPE + KV write (its intended caller order):
    the newest token's K/V and the rotated q come from that kernel, and the result must equal the
    plain entry point's and the oracle's."""
    from nano_infer_engine_b200.layers.rope import RopeScale

    g = torch.Generator().manual_seed(77)
    bs, hq, hkv, d = 16, 32, 8, 64
    lens = [1, 37, 900, 16 * 9, 2048, 333]
    B = len(lens)
    nb = sum((n + bs - 1) // bs for n in lens) + 11
    tables = _random_layout(nb, lens, bs, 77)
    kc = torch.randn(1, nb, bs, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    vc = torch.randn(1, nb, bs, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    q = torch.randn(B, hq * d, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(B, hkv * d, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(B, hkv * d, generator=g).to(torch.bfloat16).to(cuda)
    pos = torch.tensor([n - 1 for n in lens]).to(cuda)
    slots = torch.tensor([t[(n - 1) // bs] * bs + (n - 1) % bs for t, n in zip(tables, lens)]).to(cuda)
    tab = _tables_tensor(tables, cuda)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    sin, cos = RopeScale(d).sin_cos(pos, torch.bfloat16)
    outs = []
    for overlap in (True, False):
        kk, vv = kc.clone(), vc.clone()
        torch.cuda.synchronize()
        qr = ops().rope_write_kv(q, k, v, sin, cos, kk, vv, 0, slots, hq)
        outs.append(ops().paged_decode(qr, kk, vv, 0, tab, seq, overlap=overlap))
    ops().check_device_errors(cuda)
    assert torch.equal(outs[0], outs[1])
    want = oatt.paged_decode(qr.cpu(), kk.cpu(), vv.cpu(), tables, lens, 0)
    torch.testing.assert_close(outs[0].cpu().float(), want.float(), atol=2e-2, rtol=0)


@pytest.mark.parametrize("n,k", [(2048, 8192), (2048, 2048), (256, 64 * 40)])
def test_overlapped_linear_after_the_kernel_that_writes_x(cuda, n, k):
    """nie_linear_overlapped right after SiLU * up (the kernel that writes x): the weights stream
    early, x is read after that kernel; the result equals nie_linear's bit for bit."""
    g = torch.Generator().manual_seed(n + k)
    gate = torch.randn(16, k, generator=g).to(torch.bfloat16).to(cuda)
    up = torch.randn(16, k, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).to(cuda)
    outs = []
    for overlap in (True, False):
        torch.cuda.synchronize()
        act = ops().silu_mul(gate, up)
        outs.append(ops().linear_stream(act, w, overlap=overlap))
    ops().check_device_errors(cuda)
    assert torch.equal(outs[0], outs[1])
    torch.testing.assert_close(outs[0].float(), act.float() @ w.float().T, atol=2e-3, rtol=2 ** -7)


def test_bounded_wait_times_out_and_the_kernel_returns(cuda):
    """Failure path of the bounded mbarrier waits, without a fault: the timeout hook launches
    nie_linear's kernel with nothing issued on its copy ring, so every consumer wait runs out.
    The kernel must return (the call completes), raise NIE_DEV_ERR_TIMEOUT, leave zeros, and the
    next normal launch on the same context must be clean and correct."""
    from nano_infer_engine_b200 import _native

    lib = _native.lib
    g = torch.Generator().manual_seed(5)
    m, n, k = 16, 2048, 8192  # K split over a cluster: the timed-out CTAs still meet at its barrier
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).to(cuda)
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rc = lib.nie_linear_timeout_test(x.data_ptr(), k, w.data_ptr(), n, k, m, y.data_ptr(), n, _native.NIE_DTYPE_BF16,
                                     err.data_ptr(), stream, 1000)
    assert rc == 0, lib.nie_last_error()
    torch.cuda.synchronize(cuda)
    assert int(err.item()) & _native.NIE_DEV_ERR_TIMEOUT
    assert torch.equal(y, torch.zeros_like(y))
    # the context is still usable: a normal launch is clean and right
    err.zero_()
    rc = lib.nie_linear(x.data_ptr(), k, w.data_ptr(), n, k, m, y.data_ptr(), n, _native.NIE_DTYPE_BF16,
                        err.data_ptr(), stream)
    assert rc == 0, lib.nie_last_error()
    torch.cuda.synchronize(cuda)
    assert int(err.item()) == 0
    torch.testing.assert_close(y.float(), x.float() @ w.float().T, atol=1e-3, rtol=2 ** -7)
    # probe counts outside [1, 2^22] are refused on the host
    assert lib.nie_linear_timeout_test(x.data_ptr(), k, w.data_ptr(), n, k, m, y.data_ptr(), n,
                                       _native.NIE_DTYPE_BF16, err.data_ptr(), stream, 0) == _native.NIE_ERR_INVALID
