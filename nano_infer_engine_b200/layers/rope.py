"""Rotary position embeddings with the reference's fp32 frequency math.

Reference: nano_infer_engine/layers/rope.py.  The inverse frequencies and
angles are computed with the same fp32 torch operations in the same order
(plain theta scaling ``:26-75``, Llama-3 piecewise scaling ``:78-200``) and
sin/cos are cast to the activation dtype before use (``:44, :72-73``), so the
rotated q/k are bit-identical to the reference on the same device.  The
rotation pairs the two halves of the head dimension (``:6-23``).

Unlike the reference, :meth:`sin_cos` is computed once per forward pass and
shared by every layer (the values do not depend on the layer).
"""

from __future__ import annotations

import math

import torch
from torch import nn


def apply_rotary(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    """Rotate ``x [..., T, H, D]`` by per-token ``sin/cos [..., T, D/2]``."""
    half = x.shape[-1] // 2
    first, second = x[..., :half], x[..., half:]
    sin = sin.unsqueeze(-2)
    cos = cos.unsqueeze(-2)
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


class Rope(nn.Module):
    """Plain RoPE (reference layers/rope.py:26-75)."""

    def __init__(self, dim: int, theta_base: float = 500000) -> None:
        super().__init__()
        if dim % 2:
            raise ValueError("rotary dimension must be even")
        self.dim = dim
        self.theta_base = theta_base

    def inv_freq(self, device: torch.device) -> torch.Tensor:
        i = torch.arange(0, self.dim, 2, dtype=torch.float32, device=device)
        return 1 / self.theta_base ** (i / self.dim)

    def _freq_key(self) -> tuple:
        return (self.dim, self.theta_base)

    def cached_inv_freq(self, device: torch.device) -> torch.Tensor:
        """:meth:`inv_freq`, computed once per device and parameter set (it is
        the same ~10 torch ops every step otherwise).  Nothing is cached while
        a CUDA graph is being captured, so the cache never holds graph-pool
        memory."""
        cache = self.__dict__.setdefault("_inv_freq_cache", {})
        key = (device, self._freq_key())
        freq = cache.get(key)
        if freq is None:
            freq = self.inv_freq(device)
            if not (device.type == "cuda" and torch.cuda.is_current_stream_capturing()):
                cache[key] = freq
        return freq

    def sin_cos(self, positions: torch.Tensor, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        """sin/cos ``[..., T, D/2]`` for integer ``positions [..., T]`` cast to ``dtype``."""
        angles = positions.to(dtype=torch.float32)[..., None] * self.cached_inv_freq(positions.device)
        return torch.sin(angles).to(dtype), torch.cos(angles).to(dtype)

    def forward(self, x: torch.Tensor, position_offset: int = 0, position_ids: torch.Tensor | None = None):
        """Reference-compatible call on ``x [B, S, H, D]``."""
        bs, seq_len, _, head_dim = x.shape
        if head_dim != self.dim:
            raise ValueError("rotary dimension mismatch")
        if position_ids is None:
            position_ids = torch.arange(position_offset, position_offset + seq_len, device=x.device)
            position_ids = position_ids.unsqueeze(0).expand(bs, seq_len)
        elif position_ids.shape != (bs, seq_len):
            raise ValueError(f"position_ids must have shape {(bs, seq_len)}, got {tuple(position_ids.shape)}")
        sin, cos = self.sin_cos(position_ids, x.dtype)
        return apply_rotary(x, sin, cos)


class RopeScale(Rope):
    """Llama-3 frequency-scaled RoPE (reference layers/rope.py:78-200)."""

    def __init__(
        self,
        dim: int,
        theta_base: float = 500000.0,
        scaling_factor: float = 32.0,
        low_freq_factor: float = 1.0,
        high_freq_factor: float = 4.0,
        original_max_position_embeddings: int = 8192,
    ) -> None:
        super().__init__(dim, theta_base)
        self.scaling_factor = scaling_factor
        self.low_freq_factor = low_freq_factor
        self.high_freq_factor = high_freq_factor
        self.original_max_position_embeddings = original_max_position_embeddings

    def _freq_key(self) -> tuple:
        return (self.dim, self.theta_base, self.scaling_factor, self.low_freq_factor, self.high_freq_factor,
                self.original_max_position_embeddings)

    def inv_freq(self, device: torch.device) -> torch.Tensor:
        base = super().inv_freq(device)
        wavelen = 2 * math.pi / base
        orig = self.original_max_position_embeddings
        low_wavelen = orig / self.low_freq_factor
        high_wavelen = orig / self.high_freq_factor
        scaled = base / self.scaling_factor
        smooth = (orig / wavelen - self.low_freq_factor) / (self.high_freq_factor - self.low_freq_factor)
        blended = (1 - smooth) * scaled + smooth * base
        low = wavelen > low_wavelen
        high = wavelen < high_wavelen
        medium = ~(low | high)
        out = torch.where(low, scaled, base)
        return torch.where(medium, blended, out)
