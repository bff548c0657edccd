"""Pre-norm Llama decoder block (reference layers/decoder.py:7-74)."""

from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..paged_cache import PagedKVCache
from .attention import GroupedQueryAttention, apply_linear, fuse_linears, fused_weight
from .mlp import SwiGLUMLP
from .rms_norm import RmsNorm


class Llama3Decoder(nn.Module):
    def __init__(self, norm_eps, q_head_num, kv_head_num, hidden_size, mlp_inner_size, rope=None) -> None:
        super().__init__()
        self.q_head_num = q_head_num
        self.kv_head_num = kv_head_num
        self.hidden_size = hidden_size
        self.norm_eps = norm_eps
        self.inner_size = mlp_inner_size
        self.attn = GroupedQueryAttention(q_head_num, kv_head_num, hidden_size, rope)
        self.ffn = SwiGLUMLP(mlp_inner_size, hidden_size)
        self.pre_norm = RmsNorm(hidden_size, eps=norm_eps)
        self.post_norm = RmsNorm(hidden_size, eps=norm_eps)

    def step(
        self,
        normed: torch.Tensor,
        residual: torch.Tensor,
        meta: ops.RaggedMeta,
        cache: PagedKVCache,
        layer_index: int,
        sin: torch.Tensor,
        cos: torch.Tensor,
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """One block on flattened tokens whose pre-norm is already applied.

        Returns ``(mlp_out, h)`` with ``h = attn_out + residual``; the caller
        adds the two inside the next fused add + RMSNorm, which is the
        reference order (``h = attn + x``, ``out = mlp(norm(h)) + h``).
        """
        attn = self.attn.attend(normed, meta, cache, layer_index, sin, cos)
        h, normed2 = ops.add_rmsnorm(attn, residual, self.post_norm.weight, self.post_norm.eps)
        fused = fused_weight(self.ffn, ("gate_proj", "up_proj"), "_gate_up")
        if fused is not None:
            gate_up = ops.linear(normed2, fused)
            inner = self.ffn.inner_size
            gate, up = gate_up[:, :inner], gate_up[:, inner:]
        else:
            gate = self.ffn.gate_proj(normed2)
            up = self.ffn.up_proj(normed2)
        # the SiLU * up kernel just before does not write weights
        return apply_linear(self.ffn.down_proj, ops.silu_mul(gate, up), overlap=True), h

    def fuse_projections(self) -> bool:
        """Single-buffer q/k/v and gate/up weights (see ``fuse_linears``)."""
        changed = self.attn.fuse_projections()
        return fuse_linears(self.ffn, ("gate_proj", "up_proj"), "_gate_up") or changed

    def forward(self, x, k_cache=None, v_cache=None, cache_position=0, attention_mask=None, position_ids=None, *,
                paged_cache=None, layer_index=None, sequence_id="default", sequence_ids=None):
        h = self.attn(
            self.pre_norm(x),
            k_cache,
            v_cache,
            cache_position,
            attention_mask,
            position_ids,
            paged_cache=paged_cache,
            layer_index=layer_index,
            sequence_id=sequence_id,
            sequence_ids=sequence_ids,
        ) + x
        return self.ffn(self.post_norm(h)) + h

    def forward_ragged(self, x, *, paged_cache, layer_index, sequence_ids, query_start_loc, context_lengths):
        h = self.attn.forward_ragged(
            self.pre_norm(x),
            paged_cache=paged_cache,
            layer_index=layer_index,
            sequence_ids=sequence_ids,
            query_start_loc=query_start_loc,
            context_lengths=context_lengths,
        ) + x
        return self.ffn(self.post_norm(h)) + h
