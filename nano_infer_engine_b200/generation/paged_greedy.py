"""Offline greedy driver over the scheduler (reference generation/paged_greedy.py:12-91)."""

from __future__ import annotations

import torch

from ..paged_cache import PagedKVCache
from .config import GenerationConfig, RaggedGenerationOutput
from .paged_prefill import _validate_paged_prefill_inputs
from .request import RequestStatus
from .scheduler import ContinuousBatchingScheduler


@torch.inference_mode()
def paged_greedy_generate(
    model,
    prompts: tuple[torch.Tensor, ...],
    config: GenerationConfig,
    paged_cache: PagedKVCache,
    sequence_ids: tuple[str, ...],
    *,
    max_batch_size: int | None = None,
) -> RaggedGenerationOutput:
    if not config.use_cache:
        raise ValueError("paged greedy generation requires config.use_cache=True")
    if max_batch_size is not None and (
        isinstance(max_batch_size, bool) or not isinstance(max_batch_size, int) or max_batch_size <= 0
    ):
        raise ValueError("max_batch_size must be a positive integer")
    _validate_paged_prefill_inputs(prompts, paged_cache, sequence_ids)
    limit = max_batch_size or len(prompts)
    budget = paged_cache.allocator.free_block_count
    bs = paged_cache.block_size
    required = []
    for prompt, sid in zip(prompts, sequence_ids):
        blocks = (prompt.shape[1] + config.max_new_tokens - 1 + bs - 1) // bs
        if blocks > budget:
            raise ValueError(f"request cannot fit in paged cache: {sid}")
        required.append(blocks)
    if max_batch_size is None and sum(required) > budget:
        raise ValueError("not enough free blocks for paged generation")
    scheduler = ContinuousBatchingScheduler(
        model, config, paged_cache, limit, release_on_token_limit=max_batch_size is not None
    )
    requests = [scheduler.add_request(sid, prompt) for prompt, sid in zip(prompts, sequence_ids)]
    scheduler.run_until_idle()
    failed = next((r for r in requests if r.status is RequestStatus.FAILED), None)
    if failed is not None:
        raise RuntimeError(f"paged prefill failed: {failed.sequence_id}") from failed.error
    device = prompts[0].device
    return RaggedGenerationOutput(
        sequences=tuple(r.sequence for r in requests),
        generated_tokens=torch.tensor([r.generated_tokens for r in requests], dtype=torch.long, device=device),
        stopped_by_eos=torch.tensor([r.finished for r in requests], dtype=torch.bool, device=device),
    )
