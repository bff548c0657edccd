"""Grouped-query attention over the paged cache, on the sm_100a kernels.

Reference: nano_infer_engine/layers/attention.py:121-414.  Projections and
RoPE stay on torch (same op sequence as the reference); the KV slot write,
paged decode and varlen prefill attention are the library's kernels.  A
ragged step launches at most three attention-path kernels per layer: the
slot write (b), the decode kernel (c) over the requests with one query
token, and the varlen kernel (d) over the requests with more.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..paged_cache import PagedKVCache
from .rope import Rope


def fused_weight(module: nn.Module, names: tuple[str, ...], attr: str) -> torch.Tensor | None:
    """The concatenated weight of ``names`` if their parameters are still views of it.

    Reads the module dictionaries directly: this runs for every layer of every
    step, and nn.Module attribute lookups cost more than the check itself."""
    d = module.__dict__
    buf = d.get(attr)
    if buf is None:
        return None
    at = buf.data_ptr()
    step = buf.element_size()
    mods = d["_modules"]
    for name in names:
        w = mods[name]._parameters["weight"]
        if w.data_ptr() != at or w.dtype != buf.dtype:
            return None
        at += w.numel() * step
    return buf


def apply_linear(module: nn.Linear, x: torch.Tensor, *, overlap: bool = False) -> torch.Tensor:
    """``module(x)`` without nn.Module call overhead when no hook is registered.

    ``overlap``: the kernel that produced ``x`` (issued just before) does not
    write the weights, so a weight-streaming GEMM may start loading them early.
    """
    if (module._forward_hooks or module._forward_pre_hooks or nn.modules.module._global_forward_hooks
            or nn.modules.module._global_forward_pre_hooks):
        return module(x)
    params = module._parameters
    return ops.linear(x, params["weight"], params["bias"], overlap=overlap)


def fuse_linears(module: nn.Module, names: tuple[str, ...], attr: str) -> bool:
    """Concatenate the weights of bias-free Linear children ``names`` (rows) into one buffer.

    The children's ``weight`` parameters are rebound as views of the buffer,
    so ``load_state_dict`` keeps writing through to it.  Returns True if the
    buffer was built now.
    """
    if fused_weight(module, names, attr) is not None:
        return False
    linears = [getattr(module, n) for n in names]
    with torch.inference_mode(False), torch.no_grad():
        buf = torch.cat([lin.weight.detach() for lin in linears], dim=0)
        start = 0
        for lin in linears:
            rows = lin.weight.shape[0]
            lin.weight = nn.Parameter(buf[start : start + rows], requires_grad=lin.weight.requires_grad)
            start += rows
    module.__dict__[attr] = buf
    return True


class GroupedQueryAttention(nn.Module):
    """Reference attention.py:121-145 parameters (q/k/v/o projections, shared rope)."""

    def __init__(self, q_head_num: int, kv_head_num: int, hidden_size: int, rope: Rope | None = None) -> None:
        super().__init__()
        if hidden_size % q_head_num or q_head_num % kv_head_num:
            raise ValueError("hidden_size % q_head_num and q_head_num % kv_head_num must be 0")
        self.head_dim = hidden_size // q_head_num
        self.q_head_num = q_head_num
        self.hidden_size = hidden_size
        self.kv_head_num = kv_head_num
        self.group_num = q_head_num // kv_head_num
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.k_proj = nn.Linear(hidden_size, kv_head_num * self.head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, kv_head_num * self.head_dim, bias=False)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.rope = rope if rope is not None else Rope(self.head_dim)

    # ------------------------------------------------------------ kernels
    def fuse_projections(self) -> bool:
        """Store q/k/v weights in one buffer (the parameters become views of it).

        One GEMM then produces q, k and v.  Returns True when the buffer was
        (re)built, e.g. after ``.to()`` replaced the parameters.
        """
        return fuse_linears(self, ("q_proj", "k_proj", "v_proj"), "_qkv")

    def rotate_and_store(
        self,
        x: torch.Tensor,
        meta: ops.RaggedMeta,
        cache: PagedKVCache,
        layer_index: int,
        sin: torch.Tensor,
        cos: torch.Tensor,
    ) -> torch.Tensor:
        """q/k/v projections, RoPE on q and k, k/v into the cache; returns q ``[T, Hq, D]``."""
        fused = fused_weight(self, ("q_proj", "k_proj", "v_proj"), "_qkv")
        if fused is not None:
            qkv = ops.linear(x, fused)
            nq = self.q_head_num * self.head_dim
            nkv = self.kv_head_num * self.head_dim
            q, k, v = qkv[:, :nq], qkv[:, nq : nq + nkv], qkv[:, nq + nkv :]
        else:
            q = self.q_proj(x)
            k = self.k_proj(x)
            v = self.v_proj(x)
        return ops.rope_write_kv(q, k, v, sin, cos, cache.keys, cache.values, layer_index, meta.slot_mapping,
                                 self.q_head_num)

    def attend(
        self,
        x: torch.Tensor,
        meta: ops.RaggedMeta,
        cache: PagedKVCache,
        layer_index: int,
        sin: torch.Tensor,
        cos: torch.Tensor,
    ) -> torch.Tensor:
        """One layer of ragged attention for flattened ``x [T, hidden]``.

        Projections on torch, then one fused kernel rotates q/k (the
        reference's RoPE rounding) and writes k/v into the cache slots, then
        the decode and varlen attention kernels, then o_proj.
        """
        T = x.shape[0]
        q = self.rotate_and_store(x, meta, cache, layer_index, sin, cos)
        out = torch.empty_like(q)
        if meta.num_decode:
            ops.paged_decode(
                q,
                cache.keys,
                cache.values,
                layer_index,
                meta.block_tables,
                meta.seq_lens,
                out=out,
                table_rows=meta.table_rows,
                q_rows=meta.query_start_loc,
                req_list=meta.decode_list,
                num_requests=meta.num_decode,
                overlap=True,  # follows the RoPE + KV write; the metadata comes from the packing kernel
            )
        if meta.num_prefill:
            ops.varlen_attention(
                q,
                cache.keys,
                cache.values,
                layer_index,
                meta.block_tables,
                meta.seq_lens,
                meta.query_start_loc,
                meta.max_query_len,
                out=out,
                table_rows=meta.table_rows,
                req_list=meta.prefill_list,
                num_requests=meta.num_prefill,
                max_seq_len=meta.max_seq_len,
            )
        # out comes from the attention (or its combine) kernel just before: it does not write weights
        return apply_linear(self.o_proj, out.view(T, self.hidden_size), overlap=True)

    # ---------------------------------------------------- reference entry
    def forward(
        self,
        x: torch.Tensor,
        k_cache=None,
        v_cache=None,
        cache_position: int = 0,
        attention_mask: torch.Tensor | None = None,
        position_ids: torch.Tensor | None = None,
        *,
        paged_cache: PagedKVCache | None = None,
        layer_index: int | None = None,
        sequence_id: str = "default",
        sequence_ids: tuple[str, ...] | None = None,
    ) -> torch.Tensor:
        """Paged decode branch of reference attention.py:147-273.

        The contiguous-cache and dense branches of the reference (used only
        by its dense greedy path) are not part of this build.
        """
        bs, seq_len, hidden = x.shape
        if hidden != self.hidden_size:
            raise ValueError("hidden size mismatch")
        if (k_cache is None) != (v_cache is None):
            raise ValueError("k_cache and v_cache must both be provided or both be None")
        if paged_cache is not None and (k_cache is not None or v_cache is not None):
            raise ValueError("contiguous cache and paged cache cannot be used together")
        if paged_cache is None:
            raise NotImplementedError(
                "nano_infer_engine_b200 attention runs on a PagedKVCache; "
                "contiguous and cache-less attention are not provided"
            )
        if seq_len != 1:
            raise ValueError("paged attention reference currently requires seq_len=1")
        if layer_index is None:
            raise ValueError("layer_index is required for paged attention")
        if attention_mask is not None and not bool(attention_mask.all()):
            raise ValueError("paged attention reference does not support padding masks")
        if sequence_ids is None:
            if bs != 1:
                raise ValueError("sequence_ids is required for batched paged attention")
            ids = (sequence_id,)
        else:
            if not isinstance(sequence_ids, tuple):
                raise TypeError("sequence_ids must be a tuple")
            if len(sequence_ids) != bs:
                raise ValueError("sequence_ids must match the batch size")
            if any(not isinstance(s, str) or not s for s in sequence_ids):
                raise ValueError("sequence IDs must be non-empty strings")
            if len(set(sequence_ids)) != len(sequence_ids):
                raise ValueError("sequence IDs must be unique within a batch")
            ids = sequence_ids
        lengths = tuple(paged_cache.get_sequence_length(s) for s in ids)
        if position_ids is not None:
            expected = torch.tensor(lengths, dtype=torch.long, device=x.device)[:, None]
            if not torch.equal(position_ids, expected):
                raise ValueError("position_ids must match paged cache sequence lengths")
        for s, n in zip(ids, lengths):
            paged_cache._resolve_position(s, n)
        meta = paged_cache.pack(ids, lengths, (1,) * bs)
        sin, cos = self.rope.sin_cos(meta.positions, x.dtype)
        out = self.attend(x.reshape(bs, hidden), meta, paged_cache, layer_index, sin, cos)
        return out.view(bs, 1, hidden)

    def forward_ragged(
        self,
        x: torch.Tensor,
        *,
        paged_cache: PagedKVCache,
        layer_index: int,
        sequence_ids: tuple[str, ...],
        query_start_loc: torch.Tensor,
        context_lengths: tuple[int, ...],
    ) -> torch.Tensor:
        """Reference attention.py:345-414 signature (packs its own metadata)."""
        boundaries = query_start_loc.tolist()
        query_lengths = tuple(b - a for a, b in zip(boundaries, boundaries[1:]))
        for s, c, q in zip(sequence_ids, context_lengths, query_lengths):
            paged_cache._resolve_position(s, c + q - 1)
        meta = paged_cache.pack(tuple(sequence_ids), tuple(context_lengths), query_lengths)
        sin, cos = self.rope.sin_cos(meta.positions, x.dtype)
        return self.attend(x, meta, paged_cache, layer_index, sin, cos)
