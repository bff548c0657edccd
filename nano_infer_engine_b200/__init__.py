"""B200-native (sm_100a) ragged-batch attention path of the nano-infer-engine API.

Drop-in module layout: ``block_allocator``, ``paged_cache``, ``layers``,
``models.llama`` and ``generation`` mirror the reference package's modules.
The kernels live in ``libnie_b200.so`` (C ABI: ``include/nie_b200.h``).
"""

from .block_allocator import BlockAllocator
from .paged_cache import PagedKVCache, PagedKVTransfer, transfer_sequence

__all__ = ["BlockAllocator", "PagedKVCache", "PagedKVTransfer", "transfer_sequence"]
