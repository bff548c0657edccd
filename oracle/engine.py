"""Torch-CPU restatement of the reference Llama forward over a paged cache (test oracle).

Follows (paths relative to the reference's src/nano_infer_engine/):
  layers/rope.py:6-23, 26-75, 78-200   rotary embedding, fp32 angles, dtype sin/cos
  layers/rms_norm.py:25-31             fp32 RMSNorm
  layers/mlp.py:18-22                  SwiGLU
  layers/decoder.py:55-74              pre-norm residual block (ragged)
  layers/attention.py:345-414          ragged attention: write, gather, causal softmax
  models/llama.py:339-394              forward_ragged: capacity, layers, lm_head, advance
It is the checker and the timed CPU baseline, never part of the product.
"""

from __future__ import annotations

import math

import torch

from .attention import varlen_attention
from .paging import OracleTables


def inv_freq(dim: int, theta: float, rope_type: str = "default", scaling: dict | None = None) -> torch.Tensor:
    i = torch.arange(0, dim, 2, dtype=torch.float32)
    base = 1 / theta ** (i / dim)  # rope.py:33-35 (and :108)
    if rope_type == "default":
        return base
    s = scaling or {}
    factor = s.get("factor", 32.0)
    low_f = s.get("low_freq_factor", 1.0)
    high_f = s.get("high_freq_factor", 4.0)
    orig = s.get("original_max_position_embeddings", 8192)
    wavelen = 2 * math.pi / base  # rope.py:110-145
    scaled = base / factor
    smooth = (orig / wavelen - low_f) / (high_f - low_f)
    smooth_freq = (1 - smooth) * scaled + smooth * base
    is_low = wavelen > orig / low_f
    is_high = wavelen < orig / high_f
    medium = ~(is_low | is_high)
    out = torch.where(is_low, scaled, base)
    return torch.where(medium, smooth_freq, out)


def rope(x: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """x [T, H, D]; rope.py:184-198 (position_ids branch) then :6-23."""
    angles = positions.to(torch.float32)[:, None] * freqs
    sin = torch.sin(angles).to(x.dtype)[:, None, :]
    cos = torch.cos(angles).to(x.dtype)[:, None, :]
    a, b = x.chunk(2, dim=-1)
    return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    h = x.float()
    h = h / torch.sqrt(torch.mean(torch.square(h), dim=-1, keepdim=True) + eps)
    return (weight.float() * h).to(x.dtype)


class OracleCache:
    """Reference PagedKVCache storage [L, nb, bs, H, D] plus its tables."""

    def __init__(self, num_blocks, block_size, num_layers, kv_heads, head_dim, dtype) -> None:
        shape = (num_layers, num_blocks, block_size, kv_heads, head_dim)
        self.keys = torch.zeros(shape, dtype=dtype)
        self.values = torch.zeros(shape, dtype=dtype)
        self.tables = OracleTables(num_blocks, block_size)
        self.block_size = block_size

    def write(self, layer: int, sid: str, start: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """paged_cache.py:264-322 restated with index arithmetic instead of a token loop."""
        slots = torch.tensor([self.tables.slot(sid, start + j) for j in range(k.shape[0])], dtype=torch.long)
        bs = self.block_size
        self.keys[layer, slots // bs, slots % bs] = k
        self.values[layer, slots // bs, slots % bs] = v


class OracleLlama:
    """State-dict driven restatement of the reference Llama3_2 (ragged path only)."""

    def __init__(self, state: dict[str, torch.Tensor], config: dict) -> None:
        self.w = state
        self.c = config
        self.hd = config["hidden_size"] // config["q_head_num"]
        self.freqs = inv_freq(self.hd, config.get("rope_theta", 500000.0), config.get("rope_type", "llama3"),
                              config.get("rope_scaling"))
        self.lm_head = state.get("lm_head.weight", state["embed.weight"])

    def _linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return x @ self.w[name].t()

    def forward_ragged(self, ids: torch.Tensor, seq_ids: list[str], qlens: list[int], cache: OracleCache,
                       last_only: bool = False) -> torch.Tensor:
        c, hd = self.c, self.hd
        hq, hkv = c["q_head_num"], c["kv_head_num"]
        contexts = [cache.tables.lengths.get(s, 0) for s in seq_ids]
        for s, ctx, q in zip(seq_ids, contexts, qlens):  # llama.py:370-379
            cache.tables.ensure_capacity(s, ctx + q)
        positions = torch.cat([torch.arange(ctx, ctx + q) for ctx, q in zip(contexts, qlens)])
        x = self.w["embed.weight"][ids]
        T = x.shape[0]
        for layer in range(c["num_layers"]):
            p = f"decoders.{layer}."
            h = rms_norm(x, self.w[p + "pre_norm.weight"], c["norm_eps"])
            q = self._linear(h, p + "attn.q_proj.weight").view(T, hq, hd)
            k = self._linear(h, p + "attn.k_proj.weight").view(T, hkv, hd)
            v = self._linear(h, p + "attn.v_proj.weight").view(T, hkv, hd)
            q = rope(q, positions, self.freqs)
            k = rope(k, positions, self.freqs)
            start = 0
            for s, ctx, ql in zip(seq_ids, contexts, qlens):
                cache.write(layer, s, ctx, k[start : start + ql], v[start : start + ql])
                start += ql
            tables = [cache.tables.tables[s] for s in seq_ids]
            attn = varlen_attention(q, cache.keys, cache.values, tables, contexts, qlens, layer)
            h = self._linear(attn.reshape(T, hq * hd), p + "attn.o_proj.weight") + x
            m = rms_norm(h, self.w[p + "post_norm.weight"], c["norm_eps"])
            gate = self._linear(m, p + "ffn.gate_proj.weight")
            up = self._linear(m, p + "ffn.up_proj.weight")
            x = self._linear(torch.nn.functional.silu(gate) * up, p + "ffn.down_proj.weight") + h
        if last_only:
            ends = torch.tensor(qlens).cumsum(0) - 1
            x = x[ends]
        logits = rms_norm(x, self.w["final_rms.weight"], c["norm_eps"]) @ self.lm_head.t()
        for s, q in zip(seq_ids, qlens):  # llama.py:392-393
            cache.tables.advance(s, q)
        return logits
