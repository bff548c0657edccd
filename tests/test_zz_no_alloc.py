"""Allocation-free paged decode, checked against the regular entry point through the C ABI.

``nie_paged_decode_noalloc`` serves callers that cannot allocate device
memory (a host-language binding with no device allocator, or a runtime whose
memory pool forbids extra cudaMalloc/cudaFree): its split-K scratch is a
fixed array inside the library instead of a caller workspace.  This file is
collected last so that a failure here does not hide any other test.
"""

import ctypes

import pytest
import torch

from nano_infer_engine_b200 import _native

pytestmark = pytest.mark.gpu

BF16 = _native.NIE_DTYPE_BF16


def _inputs(seed, batch, max_ctx, device):
    g = torch.Generator().manual_seed(seed)
    bs = 16
    lens = torch.randint(1, max_ctx + 1, (batch,), generator=g).tolist()
    lens[0] = max_ctx  # at least one request as long as asked
    blocks = sum(-(-n // bs) for n in lens)
    nb = blocks + 9
    perm = torch.randperm(nb, generator=g)
    width = max(-(-n // bs) for n in lens)
    tables = torch.full((batch, width), -1, dtype=torch.int32)
    at = 0
    for i, n in enumerate(lens):
        k = -(-n // bs)
        tables[i, :k] = perm[at : at + k].to(torch.int32)
        at += k
    kc = torch.randn(1, nb, bs, 8, 64, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn(1, nb, bs, 8, 64, generator=g).to(torch.bfloat16).to(device)
    q = torch.randn(batch, 32, 64, generator=g).to(torch.bfloat16).to(device)
    return q, kc, vc, tables.to(device), torch.tensor(lens, dtype=torch.int32, device=device)


def _common_args(q, out, kc, vc, tables, lens):
    L, nb, bs, h, d = kc.shape
    return [q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), kc.data_ptr(), vc.data_ptr(), BF16, 0, L, nb,
            bs, h, d, q.shape[1], tables.data_ptr(), tables.stride(0), None, lens.data_ptr(), None, None,
            q.shape[0], ctypes.c_float(d ** -0.5)]


def test_noalloc_decode_matches_the_allocating_entry_point_on_consecutive_calls(cuda):
    lib = _native.lib
    stream = torch.cuda.current_stream(cuda).cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    # two calls in a row with different shapes: the second one runs on the
    # scratch contents the first one left behind
    for seed, batch, max_ctx in ((0, 24, 6000), (1, 57, 2500)):
        q, kc, vc, tables, lens = _inputs(seed, batch, max_ctx, cuda)
        want = torch.empty_like(q)
        ws_bytes = lib.nie_paged_decode_workspace_size(cuda.index or 0, batch, 32, 64)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
        rc = lib.nie_paged_decode(*_common_args(q, want, kc, vc, tables, lens), ws.data_ptr(), ws_bytes,
                                  err.data_ptr(), stream)
        assert rc == 0, lib.nie_last_error()
        got = torch.full_like(q, float("nan"))
        rc = lib.nie_paged_decode_noalloc(*_common_args(q, got, kc, vc, tables, lens), err.data_ptr(), stream)
        assert rc == 0, lib.nie_last_error()
        torch.cuda.synchronize(cuda)
        assert int(err.item()) == 0
        assert torch.isfinite(got).all()
        # same kernels, same inputs: only the scratch location differs, so the
        # results are bitwise equal
        assert torch.equal(got, want)


def test_noalloc_decode_rejects_batches_beyond_its_scratch(cuda):
    lib = _native.lib
    cap = lib.nie_paged_decode_noalloc_capacity()
    assert cap == 8 * 1024 * 1024
    batch = 4096  # needs far more than the fixed array at 32 query heads
    assert lib.nie_paged_decode_workspace_size(cuda.index or 0, batch, 32, 64) > cap
    # inputs really hold `batch` requests, so the call would stay in bounds even if it ran
    q, kc, vc, tables, lens = _inputs(2, batch, 1, cuda)
    out = torch.empty_like(q)
    args = _common_args(q, out, kc, vc, tables, lens)
    rc = lib.nie_paged_decode_noalloc(*args, None, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _native.NIE_ERR_INVALID
    assert b"scratch" in lib.nie_last_error()


def test_noalloc_decode_edge_of_its_scratch(cuda):
    """The largest batch that fits the fixed array runs (and matches the allocating
    entry point); one request more is rejected before any launch."""
    lib = _native.lib
    dev = cuda.index or 0
    cap = lib.nie_paged_decode_noalloc_capacity()
    fits = 1
    while lib.nie_paged_decode_workspace_size(dev, fits + 1, 32, 64) <= cap:
        fits += 1
    assert lib.nie_paged_decode_workspace_size(dev, fits, 32, 64) <= cap
    assert lib.nie_paged_decode_workspace_size(dev, fits + 1, 32, 64) > cap
    stream = torch.cuda.current_stream(cuda).cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q, kc, vc, tables, lens = _inputs(3, fits + 1, 40, cuda)
    # the largest batch that fits: the first `fits` requests of the inputs
    sub = (q[:fits], kc, vc, tables[:fits], lens[:fits])
    want = torch.empty_like(sub[0])
    ws_bytes = lib.nie_paged_decode_workspace_size(dev, fits, 32, 64)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    rc = lib.nie_paged_decode(*_common_args(sub[0], want, *sub[1:]), ws.data_ptr(), ws_bytes, err.data_ptr(), stream)
    assert rc == 0, lib.nie_last_error()
    got = torch.full_like(want, float("nan"))
    rc = lib.nie_paged_decode_noalloc(*_common_args(sub[0], got, *sub[1:]), err.data_ptr(), stream)
    assert rc == 0, lib.nie_last_error()
    torch.cuda.synchronize(cuda)
    assert int(err.item()) == 0
    assert torch.equal(got, want)
    # one more request: rejected, nothing launched, output untouched
    out = torch.full_like(q, float("nan"))
    rc = lib.nie_paged_decode_noalloc(*_common_args(q, out, kc, vc, tables, lens), err.data_ptr(), stream)
    assert rc == _native.NIE_ERR_INVALID
    assert b"scratch" in lib.nie_last_error()
    torch.cuda.synchronize(cuda)
    assert torch.isnan(out.float()).all()


def test_noalloc_decode_empty_batch_is_a_no_op(cuda):
    lib = _native.lib
    q, kc, vc, tables, lens = _inputs(4, 2, 20, cuda)
    out = torch.full_like(q, float("nan"))
    args = _common_args(q, out, kc, vc, tables, lens)
    args[20] = 0  # num_requests
    rc = lib.nie_paged_decode_noalloc(*args, None, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == 0, lib.nie_last_error()
    torch.cuda.synchronize(cuda)
    assert torch.isnan(out.float()).all()
