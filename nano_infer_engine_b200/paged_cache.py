"""Paged K/V storage with the reference's API, backed by the sm_100a kernels.

Reference: nano_infer_engine/paged_cache.py.  The host bookkeeping (block
tables, sequence lengths, allocator, error messages) is behaviour-identical;
what changes is where the data moves:

* every sequence also owns a row of a device-resident int32 block-table
  array (``[rows, stride]``), updated incrementally when blocks are
  allocated, so kernels resolve slots on the GPU instead of per token in
  Python (reference paged_cache.py:306-322);
* ``write`` / ``gather`` / ``export_sequence`` / ``import_sequence`` run the
  slot-write, gather and block-copy kernels (one launch each) instead of
  per-token / per-block ``copy_`` loops;
* :func:`transfer_sequence` copies a sequence straight from one pool's
  blocks into freshly allocated blocks of another pool (NVLink peer copy
  when the pools are on different GPUs), the P/D handoff of
  nano_infer_engine/generation/pd_scheduler.py:144-145 (export_sequence
  then import_sequence) without the intermediate stacked tensor.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .block_allocator import BlockAllocator


def _is_int(value: object) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def _check_sequence_id(sequence_id: object) -> None:
    if not isinstance(sequence_id, str):
        raise TypeError("sequence_id must be a string")
    if not sequence_id:
        raise ValueError("sequence_id must not be empty")


@dataclass(frozen=True)
class PagedKVTransfer:
    """Logical blocks exported from one cache (reference paged_cache.py:9-19)."""

    sequence_id: str
    sequence_length: int
    block_size: int
    num_layers: int
    kv_head_num: int
    head_dim: int
    keys: torch.Tensor
    values: torch.Tensor


class PagedKVCache:
    """Physical K/V blocks plus per-sequence block tables (reference paged_cache.py:22-374)."""

    _INITIAL_ROWS = 16
    _INITIAL_COLS = 64

    def __init__(
        self,
        num_blocks: int,
        block_size: int,
        num_layers: int,
        kv_head_num: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device | str,
    ) -> None:
        for name, value in (
            ("block_size", block_size),
            ("num_blocks", num_blocks),
            ("num_layers", num_layers),
            ("kv_head_num", kv_head_num),
            ("head_dim", head_dim),
        ):
            if not _is_int(value):
                raise TypeError(f"{name} must be an integer")
            if value <= 0:
                raise ValueError(f"{name} must be positive")

        self.block_size = block_size
        self.allocator = BlockAllocator(num_blocks)
        self.num_layers = num_layers
        self.kv_head_num = kv_head_num
        self.head_dim = head_dim
        self._block_tables: dict[str, list[int]] = {}
        self._sequence_lengths: dict[str, int] = {}

        shape = (num_layers, num_blocks, block_size, kv_head_num, head_dim)
        self.keys = torch.empty(shape, dtype=dtype, device=device)
        self.values = torch.empty(shape, dtype=dtype, device=device)

        # device block-table mirror: sequence -> row
        self._rows: dict[str, int] = {}
        self._free_rows: list[int] = []
        self._rows_used = 0
        self._table_host = torch.full((self._INITIAL_ROWS, self._INITIAL_COLS), -1, dtype=torch.int32)
        self._table_dev: torch.Tensor | None = None
        self._table_dirty = True

    # ------------------------------------------------------------ metadata
    @property
    def device(self) -> torch.device:
        return self.keys.device

    def ensure_capacity(self, sequence_id: str, required_tokens: int) -> None:
        """Own enough blocks for ``required_tokens`` (reference paged_cache.py:81-107)."""
        _check_sequence_id(sequence_id)
        if not _is_int(required_tokens):
            raise TypeError("required_tokens must be an integer")
        if required_tokens <= 0:
            raise ValueError("required_tokens must be positive")
        need = -(-required_tokens // self.block_size)
        table = self._block_tables.get(sequence_id)
        have = 0 if table is None else len(table)
        if need <= have:
            return
        new_ids = self.allocator.allocate(need - have)
        if table is None:
            self._block_tables[sequence_id] = new_ids
            self._sequence_lengths[sequence_id] = 0
            table = new_ids
            self._assign_row(sequence_id)
        else:
            table.extend(new_ids)
        self._store_row_entries(sequence_id, have, new_ids)

    def get_sequence_length(self, sequence_id: str) -> int:
        _check_sequence_id(sequence_id)
        return self._sequence_lengths.get(sequence_id, 0)

    def advance(self, sequence_id: str, token_count: int) -> None:
        """Grow the cached length after all layers wrote (reference paged_cache.py:118-134)."""
        _check_sequence_id(sequence_id)
        if not _is_int(token_count):
            raise TypeError("token_count must be an integer")
        if token_count <= 0:
            raise ValueError("token_count must be positive")
        new_length = self._sequence_lengths[sequence_id] + token_count
        self._resolve_position(sequence_id, new_length - 1)
        self._sequence_lengths[sequence_id] = new_length

    def get_block_table(self, sequence_id: str) -> tuple[int, ...]:
        _check_sequence_id(sequence_id)
        return tuple(self._block_tables[sequence_id])

    def _resolve_position(self, sequence_id: str, token_position: int) -> tuple[int, int]:
        """Logical position -> (physical block, offset) (reference paged_cache.py:240-262)."""
        if not _is_int(token_position):
            raise TypeError("token_position must be an integer")
        if token_position < 0:
            raise ValueError("token_position must be non-negative")
        table = self.get_block_table(sequence_id)
        logical, offset = divmod(token_position, self.block_size)
        if logical >= len(table):
            raise IndexError("token position exceeds allocated capacity")
        return table[logical], offset

    def release(self, sequence_id: str) -> None:
        """Free every block of a sequence (reference paged_cache.py:364-374)."""
        _check_sequence_id(sequence_id)
        ids = self._block_tables[sequence_id]
        self.allocator.free(ids)
        del self._block_tables[sequence_id]
        del self._sequence_lengths[sequence_id]
        self._release_row(sequence_id)

    # ------------------------------------------------- device table mirror
    def _assign_row(self, sequence_id: str) -> None:
        if self._free_rows:
            row = self._free_rows.pop()
        else:
            row = self._rows_used
            self._rows_used += 1
            if row >= self._table_host.shape[0]:
                self._grow_table(rows=2 * self._table_host.shape[0])
        self._rows[sequence_id] = row
        self._table_host[row].fill_(-1)
        self._table_dirty = True

    def _release_row(self, sequence_id: str) -> None:
        row = self._rows.pop(sequence_id, None)
        if row is not None:
            self._table_host[row].fill_(-1)
            self._free_rows.append(row)
            self._table_dirty = True

    def _grow_table(self, rows: int | None = None, cols: int | None = None) -> None:
        old = self._table_host
        new_rows = max(rows or 0, old.shape[0])
        new_cols = max(cols or 0, old.shape[1])
        table = torch.full((new_rows, new_cols), -1, dtype=torch.int32)
        table[: old.shape[0], : old.shape[1]] = old
        self._table_host = table
        self._table_dev = None
        self._table_dirty = True

    def reserve_table(self, rows: int, cols: int) -> None:
        """Size the block-table mirror for ``rows`` live sequences of up to
        ``cols`` blocks each, so that it is not reallocated while they run
        (a reallocation retires every captured decode graph of this cache)."""
        if rows > self._table_host.shape[0] or cols > self._table_host.shape[1]:
            self._grow_table(rows=rows, cols=cols)

    def _store_row_entries(self, sequence_id: str, start: int, ids: list[int]) -> None:
        end = start + len(ids)
        if end > self._table_host.shape[1]:
            cols = self._table_host.shape[1]
            while cols < end:
                cols *= 2
            self._grow_table(cols=cols)
        row = self._rows[sequence_id]
        self._table_host[row, start:end] = torch.tensor(ids, dtype=torch.int32)
        self._table_dirty = True

    def device_block_tables(self) -> torch.Tensor:
        """The int32 ``[rows, stride]`` device copy of all live block tables."""
        if self.device.type != "cuda":
            raise RuntimeError("nano_infer_engine_b200 kernels require a CUDA cache")
        if self._table_dev is None:
            self._table_dev = torch.empty(self._table_host.shape, dtype=torch.int32, device=self.device)
            self._table_dirty = True
        if self._table_dirty:
            rows = max(self._rows_used, 1)
            host = self._table_host[:rows].pin_memory()
            self._table_dev[:rows].copy_(host, non_blocking=True)
            self._table_dirty = False
        return self._table_dev

    def table_row(self, sequence_id: str) -> int:
        return self._rows[sequence_id]

    # ------------------------------------------------------------- packing
    def pack(
        self,
        sequence_ids: tuple[str, ...],
        context_lengths: tuple[int, ...],
        query_lengths: tuple[int, ...],
    ) -> ops.RaggedMeta:
        """Build the device metadata of one ragged step (kernel (a))."""
        rows = [self._rows[s] for s in sequence_ids]
        plan_host = torch.tensor([rows, list(context_lengths), list(query_lengths)], dtype=torch.int32)
        tables = self.device_block_tables()
        plan = plan_host.pin_memory().to(self.device, non_blocking=True)
        num_decode = sum(1 for q in query_lengths if q == 1)
        return ops.pack_ragged(
            plan,
            sum(query_lengths),
            tables,
            self.block_size,
            self.allocator.num_blocks,
            num_decode=num_decode,
            max_query_len=max(query_lengths),
            max_seq_len=max(c + q for c, q in zip(context_lengths, query_lengths)),
        )

    # ------------------------------------------------------------ data ops
    def write(self, layer_index: int, sequence_id: str, start_position: int, keys, values) -> None:
        """Store K/V rows at consecutive positions (reference paged_cache.py:264-322)."""
        if not _is_int(layer_index):
            raise TypeError("layer_index must be an integer")
        if layer_index < 0 or layer_index >= self.num_layers:
            raise IndexError("layer_index out of range")
        _check_sequence_id(sequence_id)
        if not _is_int(start_position):
            raise TypeError("start_position must be an integer")
        if start_position < 0:
            raise ValueError("start_position must be non-negative")
        if not isinstance(keys, torch.Tensor) or not isinstance(values, torch.Tensor):
            raise TypeError("keys and values must be torch.Tensor objects")
        if keys.shape != values.shape:
            raise ValueError("keys and values must have identical shapes")
        if keys.ndim != 3:
            raise ValueError("keys and values must be 3D tensors")
        token_count, kv_head_num, head_dim = keys.shape
        if token_count <= 0:
            raise ValueError("keys and values must contain at least one token")
        if kv_head_num != self.kv_head_num or head_dim != self.head_dim:
            raise ValueError("keys and values must match the cache KV head count and head dimension")
        if keys.dtype != self.keys.dtype or values.dtype != self.values.dtype:
            raise ValueError("keys and values must match the cache dtype")
        if keys.device != self.keys.device or values.device != self.values.device:
            raise ValueError("keys and values must be on the cache device")
        self._resolve_position(sequence_id, start_position + token_count - 1)
        meta = self.pack((sequence_id,), (start_position,), (token_count,))
        ops.write_kv(keys, values, self.keys, self.values, layer_index, meta.slot_mapping)

    def gather(self, layer_index: int, sequence_id: str, token_count: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Contiguous copies of the first ``token_count`` K/V rows (reference paged_cache.py:324-362)."""
        if not _is_int(layer_index):
            raise TypeError("layer_index must be an integer")
        if layer_index < 0 or layer_index >= self.num_layers:
            raise IndexError("layer_index out of range")
        _check_sequence_id(sequence_id)
        if not _is_int(token_count):
            raise TypeError("token_count must be an integer")
        if token_count <= 0:
            raise ValueError("token_count must be positive")
        self._resolve_position(sequence_id, token_count - 1)
        tables = self.device_block_tables()
        row = tables[self._rows[sequence_id]]
        return ops.gather_kv(self.keys, self.values, layer_index, row, token_count)

    def export_sequence(self, sequence_id: str) -> PagedKVTransfer:
        """Snapshot ordered by logical block, zeroed tail (reference paged_cache.py:145-180)."""
        table = self.get_block_table(sequence_id)
        length = self.get_sequence_length(sequence_id)
        if length <= 0:
            raise ValueError("cannot export an empty sequence")
        n = -(-length // self.block_size)
        shape = (self.num_layers, n, self.block_size, self.kv_head_num, self.head_dim)
        keys = torch.empty(shape, dtype=self.keys.dtype, device=self.device)
        values = torch.empty_like(keys)
        src_ids = torch.tensor(table[:n], dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
        ops.copy_blocks(
            self.keys, self.values, src_ids, keys, values, None, n, length % self.block_size, run_on=self.device
        )
        return PagedKVTransfer(
            sequence_id=sequence_id,
            sequence_length=length,
            block_size=self.block_size,
            num_layers=self.num_layers,
            kv_head_num=self.kv_head_num,
            head_dim=self.head_dim,
            keys=keys,
            values=values,
        )

    def import_sequence(self, sequence_id: str, transfer: PagedKVTransfer) -> None:
        """Copy exported blocks into new local blocks (reference paged_cache.py:182-238)."""
        _check_sequence_id(sequence_id)
        if not isinstance(transfer, PagedKVTransfer):
            raise TypeError("transfer must be a PagedKVTransfer")
        if sequence_id in self._block_tables:
            raise ValueError(f"sequence ID already exists: {sequence_id}")
        n = -(-transfer.sequence_length // self.block_size)
        expected = (self.num_layers, n, self.block_size, self.kv_head_num, self.head_dim)
        if transfer.sequence_length <= 0:
            raise ValueError("transfer sequence length must be positive")
        if (
            transfer.block_size != self.block_size
            or transfer.num_layers != self.num_layers
            or transfer.kv_head_num != self.kv_head_num
            or transfer.head_dim != self.head_dim
        ):
            raise ValueError("transfer layout does not match the destination cache")
        if transfer.keys.shape != expected:
            raise ValueError("transfer keys have an invalid shape")
        if transfer.values.shape != expected:
            raise ValueError("transfer values have an invalid shape")
        if transfer.keys.dtype != self.keys.dtype:
            raise ValueError("transfer keys must match the cache dtype")
        if transfer.values.dtype != self.values.dtype:
            raise ValueError("transfer values must match the cache dtype")

        self.ensure_capacity(sequence_id, transfer.sequence_length)
        try:
            table = self.get_block_table(sequence_id)
            dst_ids = torch.tensor(table[:n], dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
            src_device = transfer.keys.device
            if src_device != self.device:
                _order_after(self.device, src_device)
            ops.copy_blocks(
                transfer.keys.contiguous(),
                transfer.values.contiguous(),
                None,
                self.keys,
                self.values,
                dst_ids,
                n,
                0,
                run_on=self.device,
            )
            self.advance(sequence_id, transfer.sequence_length)
        except Exception:
            self.release(sequence_id)
            raise


def _order_after(waiter: torch.device, producer: torch.device) -> None:
    """Make ``waiter``'s current stream wait for ``producer``'s queued work."""
    event = torch.cuda.Event()
    event.record(torch.cuda.current_stream(producer))
    torch.cuda.current_stream(waiter).wait_event(event)


def transfer_sequence(source: PagedKVCache, destination: PagedKVCache, sequence_id: str) -> None:
    """Move one sequence's KV from ``source`` blocks into new ``destination`` blocks.

    Equivalent to ``destination.import_sequence(sequence_id,
    source.export_sequence(sequence_id))`` (including the zeroed tail of the
    last block) but copies block to block with one kernel: the prefill GPU
    writes straight into the decode GPU's pool over NVLink.  The destination
    stream is ordered after the copy, and the copy after the destination's
    queued work (freshly allocated blocks may have been read until just now).
    """
    if not isinstance(source, PagedKVCache) or not isinstance(destination, PagedKVCache):
        raise TypeError("source and destination must be PagedKVCache objects")
    if source is destination:
        raise ValueError("source and destination must be different caches")
    if (
        source.block_size != destination.block_size
        or source.num_layers != destination.num_layers
        or source.kv_head_num != destination.kv_head_num
        or source.head_dim != destination.head_dim
    ):
        raise ValueError("transfer layout does not match the destination cache")
    if source.keys.dtype != destination.keys.dtype:
        raise ValueError("transfer keys must match the cache dtype")
    _check_sequence_id(sequence_id)
    if sequence_id in destination._block_tables:
        raise ValueError(f"sequence ID already exists: {sequence_id}")
    src_table = source.get_block_table(sequence_id)
    length = source.get_sequence_length(sequence_id)
    if length <= 0:
        raise ValueError("cannot export an empty sequence")
    bs = source.block_size
    n = -(-length // bs)

    destination.ensure_capacity(sequence_id, length)
    try:
        dst_table = destination.get_block_table(sequence_id)
        run_device = source.device
        src_ids = torch.tensor(src_table[:n], dtype=torch.int32).pin_memory().to(run_device, non_blocking=True)
        dst_ids = torch.tensor(dst_table[:n], dtype=torch.int32).pin_memory().to(run_device, non_blocking=True)
        if destination.device != run_device:
            _order_after(run_device, destination.device)
        ops.copy_blocks(
            source.keys,
            source.values,
            src_ids,
            destination.keys,
            destination.values,
            dst_ids,
            n,
            length % bs,
            run_on=run_device,
        )
        if destination.device != run_device:
            _order_after(destination.device, run_device)
        destination.advance(sequence_id, length)
    except Exception:
        destination.release(sequence_id)
        raise
