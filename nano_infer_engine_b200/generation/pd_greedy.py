"""Synchronous single-request prefill/decode disaggregation (reference generation/pd_greedy.py).

The KV handoff is :func:`transfer_sequence`: one block-copy kernel from the
prefill pool straight into the decode pool (NVLink peer stores when the
pools are on different GPUs), instead of export -> stacked tensor -> per
block cross-device ``copy_`` (reference pd_greedy.py:86-87).
"""

from __future__ import annotations

import torch

from ..paged_cache import PagedKVCache, transfer_sequence
from .config import GenerationConfig, GenerationOutput
from .paged_prefill import _validate_paged_prefill_inputs, paged_prefill


def _validate_model_cache(model, cache: PagedKVCache, name: str) -> None:
    if model.embed.weight.device != cache.keys.device:
        raise ValueError(f"{name} model and cache must be on the same device")
    if model.embed.weight.dtype != cache.keys.dtype:
        raise ValueError(f"{name} model and cache must have the same dtype")
    if len(model.decoders) != cache.num_layers:
        raise ValueError(f"{name} model and cache must have the same layer count")
    if model.config.kv_head_num != cache.kv_head_num:
        raise ValueError(f"{name} model and cache must have the same KV head count")
    if model.config.head_dim != cache.head_dim:
        raise ValueError(f"{name} model and cache must have the same head dimension")


def _release_if_allocated(cache: PagedKVCache, sequence_id: str) -> None:
    if sequence_id in cache._block_tables:
        cache.release(sequence_id)


@torch.inference_mode()
def pd_greedy_generate(
    prefill_model,
    decode_model,
    input_ids: torch.Tensor,
    config: GenerationConfig,
    prefill_cache: PagedKVCache,
    decode_cache: PagedKVCache,
    sequence_id: str = "default",
) -> GenerationOutput:
    """Prefill, hand the KV over, then decode one request (reference pd_greedy.py:31-137)."""
    if not config.use_cache:
        raise ValueError("P/D generation requires config.use_cache=True")
    if input_ids.ndim != 2 or input_ids.shape[0] != 1:
        raise ValueError("input_ids must have shape (1, prompt_length)")
    if input_ids.shape[1] <= 0:
        raise ValueError("input_ids must contain at least one token")
    if not isinstance(prefill_cache, PagedKVCache):
        raise TypeError("prefill_cache must be a PagedKVCache")
    if not isinstance(decode_cache, PagedKVCache):
        raise TypeError("decode_cache must be a PagedKVCache")
    if prefill_cache is decode_cache:
        raise ValueError("prefill_cache and decode_cache must be different caches")
    _validate_model_cache(prefill_model, prefill_cache, "prefill")
    _validate_model_cache(decode_model, decode_cache, "decode")
    _validate_paged_prefill_inputs((input_ids,), prefill_cache, (sequence_id,))
    if sequence_id in decode_cache._block_tables:
        raise ValueError(f"sequence ID already exists: {sequence_id}")
    capacity = input_ids.shape[1] + config.max_new_tokens - 1
    bs = decode_cache.block_size
    if (capacity + bs - 1) // bs > decode_cache.allocator.free_block_count:
        raise ValueError("not enough free blocks in decode cache")

    device = decode_cache.keys.device
    try:
        last_logits = paged_prefill(prefill_model, (input_ids,), prefill_cache, (sequence_id,))
        transfer_sequence(prefill_cache, decode_cache, sequence_id)
        last_logits = last_logits.to(device)
    except Exception:
        _release_if_allocated(decode_cache, sequence_id)
        raise
    finally:
        _release_if_allocated(prefill_cache, sequence_id)

    sequences = input_ids.to(device)
    generated = torch.zeros(1, dtype=torch.long, device=device)
    stopped = torch.zeros(1, dtype=torch.bool, device=device)
    try:
        for step in range(config.max_new_tokens):
            next_token = last_logits.argmax(dim=-1, keepdim=True)
            sequences = torch.cat((sequences, next_token), dim=1)
            generated += 1
            if config.eos_token_id is not None:
                stopped |= next_token.squeeze(-1).eq(config.eos_token_id)
                if stopped.all():
                    break
            if step + 1 < config.max_new_tokens:
                logits = decode_model(next_token, kv_cache=decode_cache, sequence_id=sequence_id)
                last_logits = logits[:, -1]
    except Exception:
        _release_if_allocated(decode_cache, sequence_id)
        raise
    return GenerationOutput(sequences=sequences, generated_tokens=generated, stopped_by_eos=stopped)
