"""Integer restatement of the reference's paging metadata (test oracle).

Every function cites the reference line it follows
(paths relative to the reference's src/nano_infer_engine/).
"""

from __future__ import annotations


class OracleAllocator:
    """block_allocator.py:4-60: LIFO stack, fresh pool yields 0,1,2,...; free pushes reversed."""

    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self.free = list(range(num_blocks - 1, -1, -1))  # :15
        self.used: set[int] = set()

    def allocate(self, count: int) -> list[int]:  # :26-37
        if count > len(self.free):
            raise ValueError("not enough free blocks")
        out = [self.free.pop() for _ in range(count)]
        self.used.update(out)
        return out

    def release(self, ids: list[int]) -> None:  # :39-60
        for b in ids:
            if b not in self.used:
                raise ValueError(f"block is not allocated: {b}")
        for b in ids:
            self.used.remove(b)
        self.free.extend(reversed(ids))


class OracleTables:
    """paged_cache.py:81-134, 364-374: per-sequence tables and lengths."""

    def __init__(self, num_blocks: int, block_size: int) -> None:
        self.block_size = block_size
        self.alloc = OracleAllocator(num_blocks)
        self.tables: dict[str, list[int]] = {}
        self.lengths: dict[str, int] = {}

    def ensure_capacity(self, sid: str, tokens: int) -> None:  # :81-107
        need = (tokens + self.block_size - 1) // self.block_size
        have = len(self.tables.get(sid, []))
        if need > have:
            ids = self.alloc.allocate(need - have)
            if sid not in self.tables:
                self.tables[sid] = ids
                self.lengths[sid] = 0
            else:
                self.tables[sid].extend(ids)

    def advance(self, sid: str, count: int) -> None:  # :118-134
        self.lengths[sid] += count

    def release(self, sid: str) -> None:  # :364-374
        self.alloc.release(self.tables[sid])
        del self.tables[sid]
        del self.lengths[sid]

    def slot(self, sid: str, position: int) -> int:  # :240-262 (block*bs + offset)
        block = self.tables[sid][position // self.block_size]
        return block * self.block_size + position % self.block_size


def ragged_metadata(
    tables: list[list[int]], contexts: list[int], query_lengths: list[int], block_size: int
) -> dict[str, list[int]]:
    """query_start_loc (paged_prefill.py:132-143), positions (attention.py:363-376),
    slot mapping (paged_cache.py:311-322 via :240-262), last rows (paged_prefill.py:154)."""
    qsl = [0]
    for q in query_lengths:
        qsl.append(qsl[-1] + q)
    positions: list[int] = []
    slots: list[int] = []
    for table, ctx, q in zip(tables, contexts, query_lengths):
        for j in range(q):
            p = ctx + j
            positions.append(p)
            slots.append(table[p // block_size] * block_size + p % block_size)
    return {
        "query_start_loc": qsl,
        "positions": positions,
        "slot_mapping": slots,
        "seq_lens": [c + q for c, q in zip(contexts, query_lengths)],
        "last_token_index": [e - 1 for e in qsl[1:]],
        "decode_list": [i for i, q in enumerate(query_lengths) if q == 1],
        "prefill_list": [i for i, q in enumerate(query_lengths) if q != 1],
    }
