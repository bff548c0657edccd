"""Scheduler outputs (reference generation/events.py:9-33)."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .request import PagedRequest, RequestStatus


@dataclass(frozen=True)
class TokenEvent:
    sequence_id: str
    token_id: int


@dataclass(frozen=True)
class SchedulerStepOutput:
    token_events: tuple[TokenEvent, ...]
    terminal_requests: tuple[PagedRequest, ...]


@dataclass(frozen=True)
class RequestResult:
    sequence_id: str
    status: RequestStatus
    sequence: torch.Tensor
    generated_tokens: int
    stopped_by_eos: bool
    error: Exception | None
