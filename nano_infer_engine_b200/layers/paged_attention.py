"""Paged decode attention with the reference's function signatures.

Reference: nano_infer_engine/layers/paged_attention.py.  The same argument
validation (types, shapes, messages) runs on the host; the attention itself
is one launch of the sm_100a decode kernel (``nie_paged_decode``) instead of
a Python loop over blocks and sequences.
"""

from __future__ import annotations

import torch

from .. import ops


def _is_int(value: object) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def _validate_query_and_caches(query: torch.Tensor, key_cache, value_cache, ndim: int) -> None:
    if not isinstance(query, torch.Tensor):
        raise TypeError("query must be a torch.Tensor")
    if not isinstance(key_cache, torch.Tensor) or not isinstance(value_cache, torch.Tensor):
        raise TypeError("key_cache and value_cache must be torch.Tensor objects")
    if query.ndim != ndim:
        raise ValueError(f"query must be a {ndim}D tensor")
    if key_cache.ndim != 5 or value_cache.ndim != 5:
        raise ValueError("key_cache and value_cache must be 5D tensors")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache must have identical shapes")
    if query.dtype != key_cache.dtype or query.dtype != value_cache.dtype:
        raise ValueError("query and K/V caches must have the same dtype")
    if query.device != key_cache.device or query.device != value_cache.device:
        raise ValueError("query and K/V caches must be on the same device")
    if not query.is_floating_point():
        raise ValueError("query and K/V caches must use a floating-point dtype")
    if min(key_cache.shape) <= 0:
        raise ValueError("K/V cache dimensions must be positive")
    if query.shape[-1] != key_cache.shape[-1]:
        raise ValueError("query and K/V caches must have the same head dimension")
    if query.shape[-2] % key_cache.shape[3] != 0:
        raise ValueError("q_head_num must be divisible by kv_head_num")


def _validate_table(block_table, sequence_length, block_size: int, num_blocks: int) -> None:
    if not isinstance(block_table, tuple):
        raise TypeError("block_table must be a tuple")
    required = -(-sequence_length // block_size)
    if len(block_table) < required:
        raise ValueError("block_table does not cover sequence_length")
    used = block_table[:required]
    if any(not _is_int(b) for b in used):
        raise TypeError("block IDs must be integers")
    if any(b < 0 or b >= num_blocks for b in used):
        raise ValueError("block ID out of range")


def batched_paged_attention_reference(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: tuple[tuple[int, ...], ...],
    sequence_lengths: tuple[int, ...],
    layer_index: int,
) -> torch.Tensor:
    """Decode attention for ``query [B, Hq, D]`` (reference paged_attention.py:117-176).

    The name is kept so callers of the reference need no change; the work is
    a single kernel launch.
    """
    if not isinstance(query, torch.Tensor):
        raise TypeError("query must be a torch.Tensor")
    if query.ndim != 3:
        raise ValueError("query must be a 3D tensor")
    batch = query.shape[0]
    if batch <= 0:
        raise ValueError("query batch size must be positive")
    if not isinstance(block_tables, tuple):
        raise TypeError("block_tables must be a tuple")
    if not isinstance(sequence_lengths, tuple):
        raise TypeError("sequence_lengths must be a tuple")
    if len(block_tables) != batch:
        raise ValueError("block_tables must match the query batch size")
    if len(sequence_lengths) != batch:
        raise ValueError("sequence_lengths must match the query batch size")
    if any(not isinstance(t, tuple) for t in block_tables):
        raise TypeError("each block table must be a tuple")
    if any(not _is_int(n) for n in sequence_lengths):
        raise TypeError("sequence lengths must be integers")
    if any(n <= 0 for n in sequence_lengths):
        raise ValueError("sequence lengths must be positive")
    _validate_query_and_caches(query, key_cache, value_cache, 3)
    if not _is_int(layer_index):
        raise TypeError("layer_index must be an integer")
    num_layers, num_blocks, block_size = key_cache.shape[:3]
    if layer_index < 0 or layer_index >= num_layers:
        raise IndexError("layer_index out of range")
    for table, n in zip(block_tables, sequence_lengths):
        _validate_table(table, n, block_size, num_blocks)

    width = max(-(-n // block_size) for n in sequence_lengths)
    table_host = torch.full((batch, width), -1, dtype=torch.int32)
    for row, (table, n) in enumerate(zip(block_tables, sequence_lengths)):
        used = -(-n // block_size)
        table_host[row, :used] = torch.tensor(table[:used], dtype=torch.int32)
    device = query.device
    tables = table_host.pin_memory().to(device, non_blocking=True)
    lens = torch.tensor(sequence_lengths, dtype=torch.int32).pin_memory().to(device, non_blocking=True)
    return ops.paged_decode(
        query.contiguous(),
        key_cache.contiguous(),
        value_cache.contiguous(),
        layer_index,
        tables,
        lens,
    )


def paged_attention_reference(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: tuple[int, ...],
    sequence_length: int,
    layer_index: int,
) -> torch.Tensor:
    """Single-sequence form ``query [Hq, D]`` (reference paged_attention.py:4-114)."""
    _validate_query_and_caches(query, key_cache, value_cache, 2)
    if not _is_int(sequence_length):
        raise TypeError("sequence_length must be an integer")
    if sequence_length <= 0:
        raise ValueError("sequence_length must be positive")
    if not _is_int(layer_index):
        raise TypeError("layer_index must be an integer")
    if not isinstance(block_table, tuple):
        raise TypeError("block_table must be a tuple")
    return batched_paged_attention_reference(
        query.unsqueeze(0), key_cache, value_cache, (block_table,), (sequence_length,), layer_index
    )[0]
