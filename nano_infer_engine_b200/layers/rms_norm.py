"""RMSNorm computed in fp32 and cast back (reference layers/rms_norm.py:25-31)."""

from __future__ import annotations

import torch
from torch import nn


class RmsNorm(nn.Module):
    def __init__(self, normalized_shape: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.eps = eps
        self.normalized_shape = normalized_shape
        self.weight = nn.Parameter(torch.ones(normalized_shape))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dtype = x.dtype
        h = x.float()
        h = h / torch.sqrt(torch.mean(torch.square(h), dim=-1, keepdim=True) + self.eps)
        return (self.weight.float() * h).to(dtype)
