"""Prefill entry points (reference generation/paged_prefill.py).

``paged_prefill`` batches prompts of equal length into one model call per
length; ``paged_prefill_chunks`` flattens ragged chunks into one
``forward_ragged`` call.  Both keep the reference's validation, capacity
checks and rollback.  Two host-side differences, invisible to callers:

* ``query_start_loc`` is built on the host (the lengths are host values)
  and uploaded once; its host copy rides along on the tensor so this
  package's model does not read it back (reference llama.py:358 does a
  device-to-host ``tolist``);
* the model is asked for last-row logits only; models that ignore the
  request (e.g. test doubles) return full logits and are indexed as in the
  reference (paged_prefill.py:154-155).
"""

from __future__ import annotations

import torch

from ..models.llama import HOST_BOUNDARIES, LAST_ROWS_DONE, LAST_ROWS_ONLY
from ..paged_cache import PagedKVCache


def _flat_view(chunks: tuple[torch.Tensor, ...]) -> torch.Tensor | None:
    """The chunks as one 1-D tensor without a copy when they are consecutive
    pieces of one buffer (a decode step's sampled tokens), else None."""
    first = chunks[0]
    if first.stride(1) != 1:
        return None
    p = first.data_ptr()
    storage = first.untyped_storage().data_ptr()
    size = first.element_size()
    total = 0
    for c in chunks:
        if c.dtype != first.dtype or c.data_ptr() != p + total * size or c.untyped_storage().data_ptr() != storage:
            return None
        if c.shape[1] > 1 and c.stride(1) != 1:
            return None
        total += c.shape[1]
    return first.as_strided((total,), (1,))


_ONE_TOKEN_QSL: dict[tuple[torch.device, int], torch.Tensor] = {}


def _one_token_boundaries(device: torch.device, n: int) -> torch.Tensor:
    """query_start_loc of n one-token chunks (0 .. n), uploaded once per device
    and size; callers only read it."""
    qsl = _ONE_TOKEN_QSL.get((device, n))
    if qsl is None:
        qsl = torch.arange(n + 1, dtype=torch.long).to(device)
        setattr(qsl, HOST_BOUNDARIES, list(range(n + 1)))
        setattr(qsl, LAST_ROWS_ONLY, True)
        _ONE_TOKEN_QSL[(device, n)] = qsl
    return qsl


def _validate_paged_prefill_inputs(
    prompts: tuple[torch.Tensor, ...],
    paged_cache: PagedKVCache,
    sequence_ids: tuple[str, ...],
) -> None:
    """Validation without cache mutation (reference paged_prefill.py:6-46)."""
    if not isinstance(paged_cache, PagedKVCache):
        raise TypeError("paged_cache must be a PagedKVCache")
    if not isinstance(prompts, tuple):
        raise TypeError("prompts must be a tuple")
    if not isinstance(sequence_ids, tuple):
        raise TypeError("sequence_ids must be a tuple")
    if not prompts:
        raise ValueError("prompts must not be empty")
    if len(prompts) != len(sequence_ids):
        raise ValueError("prompts and sequence_ids must have the same length")
    if any(not isinstance(s, str) or not s for s in sequence_ids):
        raise ValueError("sequence IDs must be non-empty strings")
    if len(set(sequence_ids)) != len(sequence_ids):
        raise ValueError("sequence IDs must be unique")
    for prompt in prompts:
        if not isinstance(prompt, torch.Tensor):
            raise TypeError("each prompt must be a torch.Tensor")
        if prompt.ndim != 2 or prompt.shape[0] != 1:
            raise ValueError("each prompt must have shape (1, prompt_length)")
        if prompt.shape[1] <= 0:
            raise ValueError("each prompt must contain at least one token")
        if prompt.device != paged_cache.keys.device:
            raise ValueError("each prompt must be on the paged cache device")
    for s in sequence_ids:
        if s in paged_cache._block_tables:
            raise ValueError(f"sequence ID already exists: {s}")


@torch.inference_mode()
def paged_prefill(
    model,
    prompts: tuple[torch.Tensor, ...],
    paged_cache: PagedKVCache,
    sequence_ids: tuple[str, ...],
) -> torch.Tensor:
    """Prefill prompts, one batched call per distinct length (reference :49-107)."""
    _validate_paged_prefill_inputs(prompts, paged_cache, sequence_ids)
    bs = paged_cache.block_size
    if sum(-(-p.shape[1] // bs) for p in prompts) > paged_cache.allocator.free_block_count:
        raise ValueError("not enough free blocks")

    by_length: dict[int, list[int]] = {}
    for index, prompt in enumerate(prompts):
        by_length.setdefault(prompt.shape[1], []).append(index)
    rows: list[torch.Tensor | None] = [None] * len(prompts)
    try:
        for members in by_length.values():
            batch = torch.cat([prompts[i] for i in members], dim=0)
            setattr(batch, LAST_ROWS_ONLY, True)
            ids = tuple(sequence_ids[i] for i in members)
            if len(ids) == 1:
                logits = model(batch, kv_cache=paged_cache, sequence_id=ids[0])
            else:
                logits = model(batch, kv_cache=paged_cache, sequence_ids=ids)
            last = logits[:, -1]
            for j, i in enumerate(members):
                rows[i] = last[j]
    except Exception:
        for s in sequence_ids:
            try:
                paged_cache.release(s)
            except KeyError:
                pass
        raise
    if any(r is None for r in rows):
        raise RuntimeError("prefill did not produce logits for every prompt")
    return torch.stack(rows)  # type: ignore[arg-type]


@torch.inference_mode()
def paged_prefill_chunks(
    model,
    chunks: tuple[torch.Tensor, ...],
    paged_cache: PagedKVCache,
    sequence_ids: tuple[str, ...],
) -> torch.Tensor:
    """One flattened ragged call; returns each chunk's last logits (reference :110-155)."""
    if not chunks:
        raise ValueError("chunks must not be empty")
    if len(chunks) != len(sequence_ids):
        raise ValueError("chunks and sequence_ids must have the same length")
    for chunk in chunks:
        if not isinstance(chunk, torch.Tensor):
            raise TypeError("each chunk must be a torch.Tensor")
        if chunk.ndim != 2 or chunk.shape[0] != 1 or chunk.shape[1] <= 0:
            raise ValueError("each chunk must have shape (1, chunk_length)")
        if chunk.device != paged_cache.keys.device:
            raise ValueError("each chunk must be on the paged cache device")
    if len(set(sequence_ids)) != len(sequence_ids):
        raise ValueError("sequence IDs must be unique")

    flat = _flat_view(chunks)
    if flat is None:
        flat = torch.cat([c[0] for c in chunks])
    if flat.is_cuda and flat.numel() == len(chunks):
        query_start_loc = _one_token_boundaries(flat.device, len(chunks))  # a decode-only step
    else:
        boundaries = [0]
        for c in chunks:
            boundaries.append(boundaries[-1] + c.shape[1])
        query_start_loc = torch.tensor(boundaries, dtype=torch.long)
        if flat.is_cuda:
            query_start_loc = query_start_loc.pin_memory().to(flat.device, non_blocking=True)
        setattr(query_start_loc, HOST_BOUNDARIES, boundaries)
        setattr(query_start_loc, LAST_ROWS_ONLY, True)
    try:
        forward_ragged = model.forward_ragged
    except AttributeError:
        raise TypeError("model must implement forward_ragged") from None
    logits = forward_ragged(
        flat,
        kv_cache=paged_cache,
        sequence_ids=sequence_ids,
        query_start_loc=query_start_loc,
    )
    if getattr(logits, LAST_ROWS_DONE, False):
        return logits
    return logits[query_start_loc[1:] - 1]
