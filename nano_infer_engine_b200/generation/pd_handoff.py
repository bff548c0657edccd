"""The prefill -> decode hand-off that both in-process P/D drivers are built on.

A :class:`PDPair` is a prefill engine (model + paged pool) and a decode
engine (model + paged pool), possibly on two GPUs.  A hand-off moves a group
of prompts from the first to the second:

1. one ragged forward prefills every prompt of the group into the prefill
   pool (last-row logits only);
2. each request's KV blocks are copied pool to pool by the block-copy
   kernel (:func:`transfer_sequence`: NVLink peer stores when the pools sit
   on different GPUs, the zeroed tail of the last block included) into
   freshly allocated decode blocks, in group order, so the decode pool's
   block tables are the ones one-request-at-a-time hand-offs would build;
3. the prefill blocks are freed.

Whatever fails, the prefill pool keeps no block of the group, and a request
whose hand-off did not finish keeps none in the decode pool.  The reference
drivers hand requests over one at a time through an intermediate stacked
tensor (reference generation/pd_scheduler.py:136-157,
generation/pd_greedy.py:79-95, paged_cache.py:145-238); the error messages
of the checks below are the reference's (generation/pd_greedy.py:9-19).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..paged_cache import PagedKVCache, transfer_sequence
from .paged_prefill import _validate_paged_prefill_inputs, paged_prefill, paged_prefill_chunks

# (what must agree, test) for a model and the pool it runs on
_PAIRING = (
    ("be on the same device", lambda m, c: m.embed.weight.device == c.keys.device),
    ("have the same dtype", lambda m, c: m.embed.weight.dtype == c.keys.dtype),
    ("have the same layer count", lambda m, c: len(m.decoders) == c.num_layers),
    ("have the same KV head count", lambda m, c: m.config.kv_head_num == c.kv_head_num),
    ("have the same head dimension", lambda m, c: m.config.head_dim == c.head_dim),
)


def check_engine(model, cache: PagedKVCache, role: str) -> None:
    """Raise ``ValueError("<role> model and cache must ...")`` for the first mismatch."""
    for what, agrees in _PAIRING:
        if not agrees(model, cache):
            raise ValueError(f"{role} model and cache must {what}")


def blocks_for(tokens: int, block_size: int) -> int:
    return -(-tokens // block_size)


def drop(cache: PagedKVCache, sequence_id: str) -> None:
    """Free the sequence's blocks in ``cache`` if it holds any."""
    if sequence_id in cache._block_tables:
        cache.release(sequence_id)


@dataclass(frozen=True)
class PDPair:
    prefill_model: object
    decode_model: object
    prefill_cache: PagedKVCache
    decode_cache: PagedKVCache

    @classmethod
    def checked(cls, prefill_model, decode_model, prefill_cache, decode_cache) -> "PDPair":
        if not isinstance(prefill_cache, PagedKVCache):
            raise TypeError("prefill_cache must be a PagedKVCache")
        if not isinstance(decode_cache, PagedKVCache):
            raise TypeError("decode_cache must be a PagedKVCache")
        if prefill_cache is decode_cache:
            raise ValueError("prefill_cache and decode_cache must be different caches")
        check_engine(prefill_model, prefill_cache, "prefill")
        check_engine(decode_model, decode_cache, "decode")
        return cls(prefill_model, decode_model, prefill_cache, decode_cache)

    @property
    def decode_device(self) -> torch.device:
        return self.decode_cache.keys.device

    def check_new(self, sequence_id: str, prompt: torch.Tensor) -> None:
        """A fresh sequence id with a well-formed prompt on the prefill device."""
        _validate_paged_prefill_inputs((prompt,), self.prefill_cache, (sequence_id,))
        if sequence_id in self.decode_cache._block_tables:
            raise ValueError(f"sequence ID already exists: {sequence_id}")

    def forget(self, sequence_id: str) -> None:
        drop(self.prefill_cache, sequence_id)
        drop(self.decode_cache, sequence_id)

    def prefill_fits(self, prompts: list[torch.Tensor]) -> bool:
        bs = self.prefill_cache.block_size
        need = sum(blocks_for(p.shape[1], bs) for p in prompts)
        return need <= self.prefill_cache.allocator.free_block_count

    @torch.inference_mode()
    def hand_off(self, sequence_ids: list[str], prompts: list[torch.Tensor]) -> list[torch.Tensor]:
        """Prefill the group in one ragged call and move each request's KV to the
        decode pool; returns each request's last-token logits on the decode device."""
        ids = tuple(sequence_ids)
        try:
            _validate_paged_prefill_inputs(tuple(prompts), self.prefill_cache, ids)
            if hasattr(self.prefill_model, "forward_ragged"):
                logits = paged_prefill_chunks(self.prefill_model, tuple(prompts), self.prefill_cache, ids)
            else:  # a model with only the batched-prompt entry point
                logits = paged_prefill(self.prefill_model, tuple(prompts), self.prefill_cache, ids)
            for sequence_id in ids:
                transfer_sequence(self.prefill_cache, self.decode_cache, sequence_id)
            return list(logits.to(self.decode_device).unbind(0))
        except Exception:
            for sequence_id in ids:
                drop(self.decode_cache, sequence_id)
            raise
        finally:
            for sequence_id in ids:
                drop(self.prefill_cache, sequence_id)
