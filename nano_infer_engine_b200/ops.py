"""Torch-facing wrappers of the C ABI: validate, then launch on the current stream.

Every function here requires CUDA tensors and calls the sm_100a library; there
is no CPU implementation.  Shapes follow the reference's cache layout
``[num_layers, num_blocks, block_size, kv_heads, head_dim]``
(nano_infer_engine/paged_cache.py:71-79).
"""

from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
from dataclasses import dataclass
from pathlib import Path

import torch

from ._native import (
    NIE_DEV_ERR_BLOCK_RANGE,
    NIE_DEV_ERR_CAPACITY,
    NIE_DEV_ERR_INDEX_RANGE,
    NIE_DEV_ERR_SLOT_RANGE,
    NIE_DEV_ERR_TIMEOUT,
    NIE_DTYPE_BF16,
    NIE_DTYPE_F16,
    NIE_DTYPE_F32,
    NIE_ERR_UNSUPPORTED,
    check,
    lib,
)

_DTYPES = {
    torch.float32: NIE_DTYPE_F32,
    torch.bfloat16: NIE_DTYPE_BF16,
    torch.float16: NIE_DTYPE_F16,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype for the paged kernels: {dtype}") from None


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "nano_infer_engine_b200 kernels require CUDA tensors "
                f"(got a tensor on {t.device})"
            )


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(where: torch.device | torch.Tensor) -> int:
    """Handle of the current CUDA stream (the launch stream) of a device or of a tensor's device."""
    if _raw_stream is not None:
        if isinstance(where, torch.Tensor):
            return _raw_stream(where.get_device())
        return _raw_stream(where.index if where.index is not None else torch.cuda.current_device())
    device = where.device if isinstance(where, torch.Tensor) else where
    return torch.cuda.current_stream(device).cuda_stream


# Number of kernels this process has launched through the library (the fast
# decode path is two kernels: the split-K pass and the combine pass).
LAUNCHES = 0


def _count(n: int = 1) -> None:
    global LAUNCHES
    LAUNCHES += n


# ------------------------------------------------------------ device errors
_err_flags: dict[int, torch.Tensor] = {}


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR their range/timeout bits into."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    flag = _err_flags.get(index)
    if flag is None:
        flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _err_flags[index] = flag
    return flag


_ERR_NAMES = {
    NIE_DEV_ERR_BLOCK_RANGE: "block id outside the pool",
    NIE_DEV_ERR_SLOT_RANGE: "slot outside the cache",
    NIE_DEV_ERR_TIMEOUT: "bounded mbarrier wait timed out",
    NIE_DEV_ERR_CAPACITY: "token position exceeds the block table",
    NIE_DEV_ERR_INDEX_RANGE: "token id outside the vocabulary",
}


def check_device_errors(device: torch.device, *, reset: bool = True) -> None:
    """Synchronise on the flag and raise if any kernel reported a violation."""
    flag = error_flag(device)
    value = int(flag.item())
    if value:
        if reset:
            flag.zero_()
        names = [name for bit, name in _ERR_NAMES.items() if value & bit]
        raise RuntimeError(f"device-side error flag {value:#x}: {', '.join(names)}")


# ------------------------------------------------------------------ packing
@dataclass
class RaggedMeta:
    """Device metadata of one ragged step, produced by :func:`pack_ragged`."""

    query_start_loc: torch.Tensor  # int64 [R+1]
    positions: torch.Tensor  # int64 [T]
    slot_mapping: torch.Tensor  # int64 [T]
    seq_lens: torch.Tensor  # int32 [R]
    last_token_index: torch.Tensor  # int64 [R]
    token_request: torch.Tensor  # int32 [T]
    decode_list: torch.Tensor  # int32 [R]
    prefill_list: torch.Tensor  # int32 [R]
    list_counts: torch.Tensor  # int32 [2]
    table_rows: torch.Tensor  # int32 [R]
    block_tables: torch.Tensor  # int32 [rows, stride]
    num_requests: int
    num_tokens: int
    num_decode: int
    num_prefill: int
    max_query_len: int
    max_seq_len: int = 0


def pack_ragged(
    plan: torch.Tensor,
    num_tokens: int,
    block_tables: torch.Tensor,
    block_size: int,
    num_blocks: int,
    *,
    num_decode: int,
    max_query_len: int,
    max_seq_len: int = 0,
) -> RaggedMeta:
    """Expand a per-request plan ``[3, R]`` (table rows, contexts, query lengths)."""
    _require_cuda(plan, block_tables)
    if plan.dtype != torch.int32 or plan.ndim != 2 or plan.shape[0] != 3 or not plan.is_contiguous():
        raise ValueError("plan must be a contiguous int32 [3, R] tensor")
    if block_tables.dtype != torch.int32 or block_tables.ndim != 2 or not block_tables.is_contiguous():
        raise ValueError("block_tables must be a contiguous int32 [rows, stride] tensor")
    device = plan.device
    R = plan.shape[1]
    T = int(num_tokens)
    i64 = torch.empty(R + 1 + 3 * T + R, dtype=torch.int64, device=device)
    i32 = torch.empty(4 * R + T + 2, dtype=torch.int32, device=device)
    qsl = i64[: R + 1]
    positions = i64[R + 1 : R + 1 + T]
    slots = i64[R + 1 + T : R + 1 + 2 * T]
    last = i64[R + 1 + 2 * T : R + 1 + 2 * T + R]
    seq_lens = i32[:R]
    dec = i32[R : 2 * R]
    pf = i32[2 * R : 3 * R]
    tok_req = i32[3 * R : 3 * R + T]
    counts = i32[3 * R + T : 3 * R + T + 2]
    status = lib.nie_pack_ragged(
        plan.data_ptr(),
        R,
        T,
        block_tables.data_ptr(),
        block_tables.shape[1],
        block_size,
        num_blocks,
        qsl.data_ptr(),
        positions.data_ptr(),
        slots.data_ptr(),
        seq_lens.data_ptr(),
        last.data_ptr(),
        tok_req.data_ptr(),
        dec.data_ptr(),
        pf.data_ptr(),
        counts.data_ptr(),
        error_flag(device).data_ptr(),
        _stream(device),
    )
    check(status, "nie_pack_ragged")
    _count()
    return RaggedMeta(
        query_start_loc=qsl,
        positions=positions,
        slot_mapping=slots,
        seq_lens=seq_lens,
        last_token_index=last,
        token_request=tok_req,
        decode_list=dec,
        prefill_list=pf,
        list_counts=counts,
        table_rows=plan[0],
        block_tables=block_tables,
        num_requests=R,
        num_tokens=T,
        num_decode=int(num_decode),
        num_prefill=R - int(num_decode),
        max_query_len=int(max_query_len),
        max_seq_len=int(max_seq_len),
    )


# --------------------------------------------------------------- KV moves
def _cache_geometry(key_cache: torch.Tensor) -> tuple[int, int, int, int, int]:
    if key_cache.ndim != 5 or not key_cache.is_contiguous():
        raise ValueError("caches must be contiguous 5D tensors")
    L, nb, bs, h, d = key_cache.shape
    return L, nb, bs, h, d


def write_kv(
    keys: torch.Tensor,
    values: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    slot_mapping: torch.Tensor,
) -> None:
    """Scatter ``keys/values [T, H, D]`` into the cache slots (bit-exact copy)."""
    _require_cuda(keys, values, key_cache, value_cache, slot_mapping)
    L, nb, bs, h, d = _cache_geometry(key_cache)
    if keys.shape != values.shape or keys.ndim != 3 or keys.shape[1:] != (h, d):
        raise ValueError("keys/values must be [T, kv_heads, head_dim] matching the cache")
    if keys.dtype != key_cache.dtype or values.dtype != value_cache.dtype:
        raise ValueError("keys/values must match the cache dtype")
    keys = keys.contiguous()
    values = values.contiguous()
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() < keys.shape[0]:
        raise ValueError("slot_mapping must be int64 with one slot per token")
    device = key_cache.device
    status = lib.nie_write_kv(
        keys.data_ptr(),
        values.data_ptr(),
        keys.shape[0],
        key_cache.data_ptr(),
        value_cache.data_ptr(),
        dtype_code(key_cache.dtype),
        layer,
        L,
        nb,
        bs,
        h,
        d,
        slot_mapping.data_ptr(),
        error_flag(device).data_ptr(),
        _stream(device),
    )
    check(status, "nie_write_kv")
    _count()


def gather_kv(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_table: torch.Tensor,
    num_tokens: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather a sequence's first ``num_tokens`` K/V rows into contiguous tensors."""
    _require_cuda(key_cache, value_cache, block_table)
    L, nb, bs, h, d = _cache_geometry(key_cache)
    if block_table.dtype != torch.int32 or not block_table.is_contiguous():
        raise ValueError("block_table must be a contiguous int32 tensor")
    out_k = torch.empty((num_tokens, h, d), dtype=key_cache.dtype, device=key_cache.device)
    out_v = torch.empty_like(out_k)
    device = key_cache.device
    status = lib.nie_gather_kv(
        key_cache.data_ptr(),
        value_cache.data_ptr(),
        dtype_code(key_cache.dtype),
        layer,
        L,
        nb,
        bs,
        h,
        d,
        block_table.data_ptr(),
        num_tokens,
        out_k.data_ptr(),
        out_v.data_ptr(),
        error_flag(device).data_ptr(),
        _stream(device),
    )
    check(status, "nie_gather_kv")
    _count()
    return out_k, out_v


def copy_blocks(
    src_keys: torch.Tensor,
    src_values: torch.Tensor,
    src_blocks: torch.Tensor | None,
    dst_keys: torch.Tensor,
    dst_values: torch.Tensor,
    dst_blocks: torch.Tensor | None,
    num_copy_blocks: int,
    tail_valid_tokens: int,
    *,
    run_on: torch.device | None = None,
) -> None:
    """Copy logical blocks between two paged pools (see ``nie_copy_blocks``).

    ``run_on`` selects the device whose stream runs the kernel (default: the
    destination).  Source and destination may live on different GPUs; peer
    access is enabled on demand.
    """
    _require_cuda(src_keys, src_values, dst_keys, dst_values, src_blocks, dst_blocks)
    L, snb, bs, h, d = _cache_geometry(src_keys)
    L2, dnb, bs2, h2, d2 = _cache_geometry(dst_keys)
    if (L, bs, h, d) != (L2, bs2, h2, d2) or src_keys.dtype != dst_keys.dtype:
        raise ValueError("source and destination pools must share layout and dtype")
    run_device = run_on if run_on is not None else dst_keys.device
    for other in (src_keys.device, dst_keys.device):
        if other != run_device:
            enable_peer_access(run_device, other)
    with torch.cuda.device(run_device):
        status = lib.nie_copy_blocks(
            src_keys.data_ptr(),
            src_values.data_ptr(),
            snb,
            _ptr(src_blocks),
            dst_keys.data_ptr(),
            dst_values.data_ptr(),
            dnb,
            _ptr(dst_blocks),
            int(num_copy_blocks),
            int(tail_valid_tokens),
            dtype_code(src_keys.dtype),
            L,
            bs,
            h,
            d,
            error_flag(run_device).data_ptr(),
            _stream(run_device),
        )
    check(status, "nie_copy_blocks")
    _count()


def copy_blocks_from_pointers(
    src_keys_ptr: int,
    src_values_ptr: int,
    src_num_blocks: int,
    src_blocks: torch.Tensor,
    dst_keys: torch.Tensor,
    dst_values: torch.Tensor,
    dst_blocks: torch.Tensor,
    num_copy_blocks: int,
    tail_valid_tokens: int,
) -> None:
    """Pull blocks from a pool known only by device pointers (an IPC mapping of a
    peer process's cache with the destination's layout) into ``dst`` on its device."""
    _require_cuda(dst_keys, dst_values, src_blocks, dst_blocks)
    L, dnb, bs, h, d = _cache_geometry(dst_keys)
    device = dst_keys.device
    with torch.cuda.device(device):
        status = lib.nie_copy_blocks(
            src_keys_ptr,
            src_values_ptr,
            src_num_blocks,
            src_blocks.data_ptr(),
            dst_keys.data_ptr(),
            dst_values.data_ptr(),
            dnb,
            dst_blocks.data_ptr(),
            int(num_copy_blocks),
            int(tail_valid_tokens),
            dtype_code(dst_keys.dtype),
            L,
            bs,
            h,
            d,
            error_flag(device).data_ptr(),
            _stream(device),
        )
    check(status, "nie_copy_blocks")
    _count()


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """64-byte CUDA IPC handle of the allocation holding ``t`` and ``t``'s offset in it."""
    _require_cuda(t)
    handle = (ctypes.c_ubyte * 64)()
    offset = ctypes.c_uint64()
    with torch.cuda.device(t.device):
        check(lib.nie_ipc_export(t.data_ptr(), handle, ctypes.byref(offset)), "nie_ipc_export")
    return bytes(handle), int(offset.value)


def ipc_import(handle: bytes, offset: int, device: torch.device) -> tuple[int, int]:
    """Map a peer process's allocation on ``device``; returns (pointer, mapping base)."""
    buf = (ctypes.c_ubyte * 64).from_buffer_copy(handle)
    ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
    with torch.cuda.device(device):
        check(lib.nie_ipc_import(buf, offset, ctypes.byref(ptr), ctypes.byref(base)), "nie_ipc_import")
    return int(ptr.value), int(base.value)


def ipc_close(base: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        check(lib.nie_ipc_close(base), "nie_ipc_close")


_peer_enabled: set[tuple[int, int]] = set()


def enable_peer_access(device: torch.device, peer: torch.device) -> None:
    key = (device.index, peer.index)
    if key in _peer_enabled:
        return
    check(lib.nie_enable_peer_access(device.index, peer.index), "nie_enable_peer_access")
    _peer_enabled.add(key)


# --------------------------------------------------------------- attention
_workspaces: dict[int, torch.Tensor] = {}


def decode_workspace(device: torch.device, num_requests: int, q_heads: int, head_dim: int) -> torch.Tensor:
    """Reusable split-K scratch for :func:`paged_decode` on ``device``."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    need = int(lib.nie_paged_decode_workspace_size(index, num_requests, q_heads, head_dim))
    ws = _workspaces.get(index)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", index))
        _workspaces[index] = ws
    return ws


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    table_rows: torch.Tensor | None = None,
    q_rows: torch.Tensor | None = None,
    req_list: torch.Tensor | None = None,
    num_requests: int | None = None,
    scale: float | None = None,
    overlap: bool = False,
) -> torch.Tensor:
    """Single-token paged attention for ``query [rows, q_heads, head_dim]``.

    ``overlap`` launches through ``nie_paged_decode_overlapped``: the kernel may
    start before the previous kernel on the stream ends, so that kernel must not
    have written ``block_tables``, ``seq_lens``, ``table_rows``, ``q_rows`` or
    ``req_list`` (it may have written the query and the caches).
    """
    _require_cuda(query, key_cache, value_cache, block_tables, seq_lens, table_rows, q_rows, req_list)
    L, nb, bs, h, d = _cache_geometry(key_cache)
    if query.ndim != 3 or query.shape[2] != d or query.stride(2) != 1 or query.stride(1) != d:
        raise ValueError("query must be [rows, q_heads, head_dim] with contiguous rows")
    if query.dtype != key_cache.dtype:
        raise ValueError("query and caches must share a dtype")
    if block_tables.dtype != torch.int32 or block_tables.ndim != 2 or block_tables.stride(1) != 1:
        raise ValueError("block_tables must be int32 [rows, stride] with contiguous rows")
    if seq_lens.dtype != torch.int32:
        raise ValueError("seq_lens must be int32")
    R = int(num_requests if num_requests is not None else seq_lens.numel())
    hq = query.shape[1]
    if out is None:
        out = torch.empty_like(query)
    device = query.device
    ws = decode_workspace(device, max(R, 1), hq, d)
    status = (lib.nie_paged_decode_overlapped if overlap else lib.nie_paged_decode)(
        query.data_ptr(),
        query.stride(0),
        out.data_ptr(),
        out.stride(0),
        key_cache.data_ptr(),
        value_cache.data_ptr(),
        dtype_code(query.dtype),
        layer,
        L,
        nb,
        bs,
        h,
        d,
        hq,
        block_tables.data_ptr(),
        block_tables.stride(0),
        _ptr(table_rows),
        seq_lens.data_ptr(),
        _ptr(q_rows),
        _ptr(req_list),
        R,
        float(d**-0.5 if scale is None else scale),
        ws.data_ptr(),
        ws.numel(),
        error_flag(device).data_ptr(),
        _stream(device),
    )
    check(status, "nie_paged_decode")
    _count(decode_launch_count(query.dtype, bs, h, d, hq))
    return out


def varlen_attention(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    query_start_loc: torch.Tensor,
    max_query_len: int,
    *,
    out: torch.Tensor | None = None,
    table_rows: torch.Tensor | None = None,
    req_list: torch.Tensor | None = None,
    num_requests: int | None = None,
    scale: float | None = None,
    max_seq_len: int | None = None,
) -> torch.Tensor:
    """Causal varlen attention of ragged query rows over the paged cache.

    ``max_seq_len`` (a host bound on every ``seq_lens`` entry) lets the
    tensor-core kernel split long key ranges across CTAs; without it each
    query tile walks all of its keys in one CTA.
    """
    _require_cuda(query, key_cache, value_cache, block_tables, seq_lens, query_start_loc, table_rows, req_list)
    L, nb, bs, h, d = _cache_geometry(key_cache)
    if query.ndim != 3 or query.shape[2] != d or query.stride(2) != 1 or query.stride(1) != d:
        raise ValueError("query must be [rows, q_heads, head_dim] with contiguous rows")
    if query_start_loc.dtype != torch.int64:
        raise ValueError("query_start_loc must be int64")
    R = int(num_requests if num_requests is not None else seq_lens.numel())
    hq = query.shape[1]
    if out is None:
        out = torch.empty_like(query)
    if out.stride(0) != query.stride(0):
        raise ValueError("out must share the query row stride")
    device = query.device
    msl = int(max_seq_len or 0)
    need = int(lib.nie_varlen_workspace_size(R, int(max_query_len), msl, hq))
    ws = varlen_workspace(device, need) if need else None
    status = lib.nie_varlen_attention(
        query.data_ptr(),
        out.data_ptr(),
        query.stride(0),
        query.shape[0],
        key_cache.data_ptr(),
        value_cache.data_ptr(),
        dtype_code(query.dtype),
        layer,
        L,
        nb,
        bs,
        h,
        d,
        hq,
        block_tables.data_ptr(),
        block_tables.stride(0),
        _ptr(table_rows),
        seq_lens.data_ptr(),
        query_start_loc.data_ptr(),
        _ptr(req_list),
        R,
        int(max_query_len),
        msl,
        float(d**-0.5 if scale is None else scale),
        _ptr(ws),
        0 if ws is None else ws.numel(),
        error_flag(device).data_ptr(),
        _stream(device),
    )
    check(status, "nie_varlen_attention")
    _count()
    return out


_varlen_workspaces: dict[int, torch.Tensor] = {}


def varlen_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Reusable split-key scratch of the tensor-core varlen kernel on ``device``."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    ws = _varlen_workspaces.get(index)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", index))
        _varlen_workspaces[index] = ws
    return ws


# ------------------------------------------------- decode-size projections
# Route projections with at most LINEAR_MAX_ROWS rows (decode steps) through
# nie_linear; False sends every projection to torch's cuBLAS GEMM.
STREAM_LINEAR = True
LINEAR_MAX_ROWS = 16


def linear_eligible(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """True when :func:`linear` runs ``x @ weight.T`` on the weight-streaming kernel.

    Taken for K >= N (o_proj, down_proj), where the kernel's K split over a
    cluster beats the library GEMM (B200, CUDA graphs, 16 rows: o_proj 4.6 vs
    5.5 us, down_proj 9.6 vs 12.9 us); for K < N (q/k/v, gate/up) the library
    GEMM is faster.

    Routing q/k/v here as well would make every kernel between the packing
    kernel and the attention a dependent launch; the overlapped decode reads
    its metadata before waiting and relies on the plain cuBLAS q/k/v launch to
    end that chain (see ``nie_paged_decode_overlapped`` in the C header): such
    a change must move the decode's metadata reads after its wait.
    """
    return (
        STREAM_LINEAR
        and weight.ndim == 2
        and weight.shape[1] >= weight.shape[0]
        and x.is_cuda
        and x.dtype == torch.bfloat16
        and weight.dtype == torch.bfloat16
        and x.ndim == 2
        and 0 < x.shape[0] <= LINEAR_MAX_ROWS
        and weight.ndim == 2
        and weight.shape[0] % 128 == 0
        and weight.shape[1] % 64 == 0
        and x.shape[1] == weight.shape[1]
        and x.stride(1) == 1
        and x.stride(0) % 8 == 0
        and weight.is_contiguous()
        and x.data_ptr() % 16 == 0
        and weight.data_ptr() % 16 == 0
    )


def linear(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, overlap: bool = False
) -> torch.Tensor:
    """``torch.nn.functional.linear(x, weight, bias)``; decode-size bf16 batches with K >= N
    stream the weights through ``nie_linear`` (fp32 accumulation, one rounding).  ``overlap``:
    see :func:`linear_stream`."""
    if bias is not None or not linear_eligible(x, weight):
        return torch.nn.functional.linear(x, weight, bias)
    return linear_stream(x, weight, overlap=overlap)


def linear_stream(x: torch.Tensor, weight: torch.Tensor, *, overlap: bool = False) -> torch.Tensor:
    """``x @ weight.T`` on ``nie_linear`` for any shape it takes (``x`` bf16 [m <= 16, k],
    ``weight`` contiguous bf16 [n, k], n and k multiples of 64); torch otherwise.

    ``overlap`` (``nie_linear_overlapped``) starts loading the weights before the previous
    kernel on the stream has finished: that kernel must not write ``weight``.
    """
    _require_cuda(x, weight)
    n, k = weight.shape
    m = x.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    status = (lib.nie_linear_overlapped if overlap else lib.nie_linear)(
        x.data_ptr(), x.stride(0), weight.data_ptr(), n, k, m, y.data_ptr(), n, NIE_DTYPE_BF16,
        error_flag(x.device).data_ptr(), _stream(x),
    )
    if status == NIE_ERR_UNSUPPORTED:  # e.g. more tiles than SMs: the library GEMM streams those well
        return torch.nn.functional.linear(x, weight)
    check(status, "nie_linear")
    _count()
    return y


# ----------------------------------------------------- fused elementwise
def add_rmsnorm(
    x: torch.Tensor,
    residual: torch.Tensor | None,
    weight: torch.Tensor,
    eps: float,
    *,
    want_sum: bool = True,
) -> tuple[torch.Tensor | None, torch.Tensor]:
    """``(x + residual, rmsnorm(x + residual) * weight)`` over the last dim, torch rounding."""
    _require_cuda(x, residual, weight)
    hidden = x.shape[-1]
    x = x.contiguous()
    if residual is not None:
        residual = residual.contiguous()
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("residual must match x")
    rows = x.numel() // hidden
    out = torch.empty_like(x)
    total = torch.empty_like(x) if (want_sum and residual is not None) else None
    status = lib.nie_add_rmsnorm(
        x.data_ptr(),
        _ptr(residual),
        weight.data_ptr(),
        float(eps),
        rows,
        hidden,
        dtype_code(x.dtype),
        _ptr(total),
        out.data_ptr(),
        _stream(x),
    )
    check(status, "nie_add_rmsnorm")
    _count()
    return (total if residual is not None else x), out


def rope_write_kv(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    slot_mapping: torch.Tensor,
    q_heads: int,
) -> torch.Tensor:
    """Rotate q/k (rows ``[T, heads*D]`` with a row stride) and write k/v to the cache slots.

    Returns the rotated queries as ``[T, q_heads, D]``.
    """
    _require_cuda(q, k, v, sin, cos, key_cache, value_cache, slot_mapping)
    L, nb, bs, h, d = _cache_geometry(key_cache)
    T = q.shape[0]
    for t, width in ((q, q_heads * d), (k, h * d), (v, h * d)):
        if t.ndim != 2 or t.shape[1] != width or t.stride(1) != 1:
            raise ValueError("q/k/v must be [T, heads*head_dim] with unit inner stride")
    if sin.shape != (T, d // 2) or not sin.is_contiguous() or not cos.is_contiguous():
        raise ValueError("sin/cos must be contiguous [T, head_dim/2]")
    q_out = torch.empty((T, q_heads, d), dtype=q.dtype, device=q.device)
    status = lib.nie_rope_write_kv(
        q.data_ptr(),
        q.stride(0),
        k.data_ptr(),
        k.stride(0),
        v.data_ptr(),
        v.stride(0),
        sin.data_ptr(),
        cos.data_ptr(),
        T,
        q_heads,
        h,
        d,
        q_out.data_ptr(),
        key_cache.data_ptr(),
        value_cache.data_ptr(),
        dtype_code(q.dtype),
        layer,
        L,
        nb,
        bs,
        slot_mapping.data_ptr(),
        error_flag(q.device).data_ptr(),
        _stream(q),
    )
    check(status, "nie_rope_write_kv")
    _count()
    return q_out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with torch's rounding, rows ``[T, inner]`` (row strides allowed)."""
    _require_cuda(gate, up)
    if gate.shape != up.shape or gate.ndim != 2 or gate.stride(1) != 1 or up.stride(1) != 1:
        raise ValueError("gate/up must be matching [T, inner] with unit inner stride")
    out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    status = lib.nie_silu_mul(
        gate.data_ptr(),
        gate.stride(0),
        up.data_ptr(),
        up.stride(0),
        out.data_ptr(),
        gate.shape[0],
        gate.shape[1],
        dtype_code(gate.dtype),
        _stream(gate),
    )
    check(status, "nie_silu_mul")
    _count()
    return out


# ----------------------------------------------------- embedding / sampling
def embed_rows(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """``table[ids]`` for int64 token ids ``[T]`` (the nn.Embedding lookup), bit-exact."""
    _require_cuda(ids, table)
    if ids.dtype != torch.int64 or ids.ndim != 1:
        raise ValueError("ids must be a 1-D int64 tensor")
    if table.ndim != 2 or not table.is_contiguous():
        raise ValueError("table must be a contiguous [vocab, hidden] tensor")
    ids = ids.contiguous()
    out = torch.empty((ids.shape[0], table.shape[1]), dtype=table.dtype, device=table.device)
    status = lib.nie_embed_rows(
        ids.data_ptr(),
        ids.shape[0],
        table.data_ptr(),
        table.shape[0],
        table.shape[1],
        dtype_code(table.dtype),
        out.data_ptr(),
        error_flag(table.device).data_ptr(),
        _stream(table),
    )
    check(status, "nie_embed_rows")
    _count()
    return out


def embed_eligible(table: torch.Tensor) -> bool:
    return table.is_cuda and table.dtype in _DTYPES and table.is_contiguous() and (
        table.shape[1] * table.element_size()) % 16 == 0 and table.data_ptr() % 16 == 0


_argmax_ws: dict[int, torch.Tensor] = {}
ARGMAX_MAX_ROWS = 4096


def argmax_rows(logits: torch.Tensor) -> torch.Tensor:
    """``logits.argmax(dim=-1)`` for ``[R, V]`` rows (R <= 4096): first index of the
    maximum, NaN ranking highest, as torch.argmax.  One launch; int64 ``[R]``."""
    _require_cuda(logits)
    if logits.ndim != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [rows, cols] with unit inner stride")
    rows, cols = logits.shape
    if rows > ARGMAX_MAX_ROWS:
        raise ValueError(f"at most {ARGMAX_MAX_ROWS} rows")
    index = logits.device.index if logits.device.index is not None else torch.cuda.current_device()
    ws = _argmax_ws.get(index)
    if ws is None:
        # fixed layout, zeroed once; CUDA graphs may capture its address
        ws = torch.zeros(int(lib.nie_argmax_workspace_size()), dtype=torch.uint8, device=logits.device)
        _argmax_ws[index] = ws
    out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    status = lib.nie_argmax_rows(
        logits.data_ptr(),
        rows,
        cols,
        logits.stride(0),
        dtype_code(logits.dtype),
        out.data_ptr(),
        ws.data_ptr(),
        ws.numel(),
        _stream(logits),
    )
    check(status, "nie_argmax_rows")
    _count()
    return out


# ------------------------------------------------------ layer-loop extension
_LAYER_LOOP_PATH = Path(__file__).resolve().parent / "_nie_torch_ext.so"
_layer_loop: object = None


def layer_loop_ext():
    """The torch C++ extension whose ``run_layers`` drives every decoder layer of
    a ragged step in one call (same kernels and cuBLAS GEMMs as the Python
    loop), or None when it has not been built (``_build.build_ext``).  A file
    that exists but does not load (built against another torch) raises."""
    global _layer_loop
    if _layer_loop is None:
        if not _LAYER_LOOP_PATH.exists():
            _layer_loop = False
        else:
            loader = importlib.machinery.ExtensionFileLoader("_nie_torch_ext", str(_LAYER_LOOP_PATH))
            spec = importlib.util.spec_from_loader("_nie_torch_ext", loader)
            module = importlib.util.module_from_spec(spec)
            loader.exec_module(module)
            _layer_loop = module
    return _layer_loop or None


def decode_launch_count(dtype: torch.dtype, block_size: int, kv_heads: int, head_dim: int, q_heads: int) -> int:
    """Kernels one :func:`paged_decode` call launches (split-K kernel + combine, or the generic one)."""
    fast = dtype == torch.bfloat16 and head_dim == 64 and block_size == 16 and q_heads // kv_heads <= 16 and kv_heads <= 16
    return 2 if fast else 1
