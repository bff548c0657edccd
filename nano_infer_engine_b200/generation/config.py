"""Generation settings (reference generation/config.py:7-50)."""

from __future__ import annotations

from dataclasses import dataclass

import torch


def _optional_positive_int(name: str, value: object) -> None:
    if value is None:
        return
    if not isinstance(value, int) or isinstance(value, bool):
        raise TypeError(f"{name} must be an integer or None")
    if value <= 0:
        raise ValueError(f"{name} must be positive")


@dataclass(frozen=True)
class GenerationConfig:
    max_new_tokens: int = 20
    eos_token_id: int | None = None
    use_cache: bool = True
    prefill_chunk_size: int | None = None
    max_prefill_tokens_per_step: int | None = None

    def __post_init__(self) -> None:
        if self.max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        _optional_positive_int("prefill_chunk_size", self.prefill_chunk_size)
        _optional_positive_int("max_prefill_tokens_per_step", self.max_prefill_tokens_per_step)
        if self.max_prefill_tokens_per_step is not None and self.prefill_chunk_size is None:
            raise ValueError("max_prefill_tokens_per_step requires prefill_chunk_size")


@dataclass
class GenerationOutput:
    sequences: torch.Tensor
    generated_tokens: torch.Tensor
    stopped_by_eos: torch.Tensor


@dataclass
class RaggedGenerationOutput:
    sequences: tuple[torch.Tensor, ...]
    generated_tokens: torch.Tensor
    stopped_by_eos: torch.Tensor
