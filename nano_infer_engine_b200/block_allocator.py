"""Host-side KV block allocator, behaviour-identical to the reference.

Reference: nano_infer_engine/block_allocator.py:4-60.  Allocation order is
part of the contract (block tables, and therefore slot mappings, must be
bit-exact): a fresh pool hands out 0, 1, 2, ...; ``free`` validates every id
before mutating state and makes freed ids come back in the order they were
passed (the stack receives them reversed).
"""

from __future__ import annotations

from collections.abc import Iterable


def _is_int(value: object) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


class BlockAllocator:
    """LIFO allocator of physical KV block ids (reference block_allocator.py:4-60)."""

    def __init__(self, num_blocks: int) -> None:
        if not _is_int(num_blocks):
            raise TypeError("num_blocks must be an integer")
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        # Stack of free ids; the top of the stack (end of the list) is the
        # next id handed out, so a fresh pool yields 0, 1, 2, ...
        self._stack: list[int] = list(range(num_blocks))[::-1]
        self._owned: set[int] = set()

    @property
    def free_block_count(self) -> int:
        return len(self._stack)

    @property
    def allocated_block_count(self) -> int:
        return len(self._owned)

    def allocate(self, block_count: int = 1) -> list[int]:
        """Pop ``block_count`` ids (reference block_allocator.py:26-37)."""
        if not _is_int(block_count):
            raise TypeError("block_count must be an integer")
        if block_count <= 0:
            raise ValueError("block_count must be positive")
        if block_count > len(self._stack):
            raise ValueError("not enough free blocks")
        taken = self._stack[-block_count:][::-1]
        del self._stack[-block_count:]
        self._owned.update(taken)
        return taken

    def free(self, block_ids: Iterable[int]) -> None:
        """Return ids atomically (reference block_allocator.py:39-60)."""
        ids = list(block_ids)
        if not all(_is_int(b) for b in ids):
            raise TypeError("block IDs must be integers")
        if len(set(ids)) != len(ids):
            raise ValueError("cannot free the same block more than once")
        for b in ids:
            if b < 0 or b >= self.num_blocks:
                raise ValueError(f"block ID out of range: {b}")
            if b not in self._owned:
                raise ValueError(f"block is not allocated: {b}")
        self._owned.difference_update(ids)
        # Push in reverse so the next allocate() returns them in given order.
        self._stack.extend(ids[::-1])
