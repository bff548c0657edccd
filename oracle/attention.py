"""Torch-CPU restatement of the reference's paged attention (test oracle).

Rounding sequence of the reference (layers/paged_attention.py:95-114 and
layers/attention.py:395-411): scores are a ``dtype`` matmul output, scaled in
``dtype``; softmax runs in fp32; probabilities are cast to ``dtype``; the PV
product is a ``dtype`` matmul.  Inputs are CPU tensors.
"""

from __future__ import annotations

import torch


def gather_sequence(cache: torch.Tensor, layer: int, table: list[int], length: int) -> torch.Tensor:
    """paged_cache.py:324-362: logical-order rows [length, H, D] of one sequence."""
    bs = cache.shape[2]
    blocks = torch.tensor(table[: (length + bs - 1) // bs], dtype=torch.long)
    rows = cache[layer, blocks].reshape(-1, cache.shape[3], cache.shape[4])
    return rows[:length]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    """q [Hq, Tq, D], k/v [Hq, Tk, D] (already GQA-expanded) -> [Hq, Tq, D]."""
    scale = q.shape[-1] ** (-0.5)
    scores = q @ k.transpose(-1, -2) * scale
    if mask is not None:
        scores = scores.masked_fill(mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    return probs.to(v.dtype) @ v


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    tables: list[list[int]],
    seq_lens: list[int],
    layer: int,
) -> torch.Tensor:
    """paged_attention.py:117-176: query [B, Hq, D] attends to all cached tokens."""
    group = query.shape[1] // key_cache.shape[3]
    out = []
    for b, (table, n) in enumerate(zip(tables, seq_lens)):
        k = gather_sequence(key_cache, layer, table, n).repeat_interleave(group, dim=1).transpose(0, 1)
        v = gather_sequence(value_cache, layer, table, n).repeat_interleave(group, dim=1).transpose(0, 1)
        out.append(_attend(query[b].unsqueeze(1), k, v, None)[:, 0])
    return torch.stack(out)


def varlen_attention(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    tables: list[list[int]],
    contexts: list[int],
    query_lengths: list[int],
    layer: int,
) -> torch.Tensor:
    """attention.py:392-413 after the write: query [T, Hq, D] -> [T, Hq, D], causal per request."""
    group = query.shape[1] // key_cache.shape[3]
    outs = []
    start = 0
    for table, ctx, ql in zip(tables, contexts, query_lengths):
        n = ctx + ql
        k = gather_sequence(key_cache, layer, table, n).repeat_interleave(group, dim=1).transpose(0, 1)
        v = gather_sequence(value_cache, layer, table, n).repeat_interleave(group, dim=1).transpose(0, 1)
        q = query[start : start + ql].transpose(0, 1)
        qpos = torch.arange(ctx, n)[:, None]
        kpos = torch.arange(n)[None, :]
        outs.append(_attend(q, k, v, kpos > qpos).transpose(0, 1))
        start += ql
    return torch.cat(outs, dim=0)
