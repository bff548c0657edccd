"""SwiGLU feed-forward block (reference layers/mlp.py:7-22); dense GEMMs stay on torch."""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


class SwiGLUMLP(nn.Module):
    def __init__(self, inner_size: int, hidden_size: int) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.inner_size = inner_size
        self.down_proj = nn.Linear(inner_size, hidden_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, inner_size, bias=False)
        self.gate_proj = nn.Linear(hidden_size, inner_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
