"""Synchronous prefill/decode disaggregation of one request (the reference's
generation/pd_greedy.py API).

The request is handed over with :class:`PDPair` (one ragged prefill, a
block-to-block KV copy into the decode pool, prefill blocks freed), then
decoded greedily on the decode engine.  Generated ids go into a preallocated
device row and each next input is a view of it: no growing ``torch.cat`` per
token, and no device-to-host read per token unless an EOS id is configured
(only then must each token be inspected before the next forward).
"""

from __future__ import annotations

import torch

from ..paged_cache import PagedKVCache
from .config import GenerationConfig, GenerationOutput
from .pd_handoff import PDPair, blocks_for, drop


def _check_call(input_ids: torch.Tensor, config: GenerationConfig) -> None:
    if not config.use_cache:
        raise ValueError("P/D generation requires config.use_cache=True")
    if input_ids.ndim != 2 or input_ids.shape[0] != 1:
        raise ValueError("input_ids must have shape (1, prompt_length)")
    if input_ids.shape[1] <= 0:
        raise ValueError("input_ids must contain at least one token")


def _greedy_decode(decode_model, cache: PagedKVCache, sequence_id: str, prompt: torch.Tensor,
                   first_logits: torch.Tensor, config: GenerationConfig) -> GenerationOutput:
    dev = cache.keys.device
    start = prompt.shape[1]
    row = torch.empty((1, start + config.max_new_tokens), dtype=prompt.dtype, device=dev)
    row[:, :start].copy_(prompt)
    eos = config.eos_token_id
    logits = first_logits.reshape(1, -1)
    produced, hit_eos = 0, False
    while produced < config.max_new_tokens:
        at = start + produced
        row[:, at : at + 1] = logits.argmax(dim=-1, keepdim=True)
        produced += 1
        if eos is not None and int(row[0, at]) == eos:
            hit_eos = True
            break
        if produced < config.max_new_tokens:
            logits = decode_model(row[:, at : at + 1], kv_cache=cache, sequence_id=sequence_id)[:, -1]
    return GenerationOutput(
        sequences=row[:, : start + produced],
        generated_tokens=torch.full((1,), produced, dtype=torch.long, device=dev),
        stopped_by_eos=torch.full((1,), hit_eos, dtype=torch.bool, device=dev),
    )


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
    """Prefill on the prefill engine, hand the KV over, decode greedily on the decode engine.

    The prefill pool ends with no blocks of the request.  On success the decode
    pool keeps the sequence (the caller may inspect, continue or release it);
    on any failure it keeps nothing of it.
    """
    _check_call(input_ids, config)
    pair = PDPair.checked(prefill_model, decode_model, prefill_cache, decode_cache)
    pair.check_new(sequence_id, input_ids)
    worst_case = blocks_for(input_ids.shape[1] + config.max_new_tokens - 1, decode_cache.block_size)
    if worst_case > decode_cache.allocator.free_block_count:
        raise ValueError("not enough free blocks in decode cache")
    (first_logits,) = pair.hand_off([sequence_id], [input_ids])
    try:
        return _greedy_decode(decode_model, decode_cache, sequence_id, input_ids.to(pair.decode_device),
                              first_logits, config)
    except Exception:
        drop(decode_cache, sequence_id)
        raise
