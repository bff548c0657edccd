"""Per-request generation state (reference generation/request.py:7-34).

``sequence`` is materialised lazily: generated token ids are kept in a host
list and concatenated to the prompt on first access, instead of one device
``torch.cat`` per request per step.  Before any token is generated it *is*
the prompt tensor, as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum

import torch


class RequestStatus(str, Enum):
    PENDING = "pending"
    PREFILLING = "prefilling"
    ACTIVE = "active"
    COMPLETED = "completed"
    FAILED = "failed"
    CANCELLED = "cancelled"


@dataclass
class PagedRequest:
    sequence_id: str
    prompt: torch.Tensor
    generated_tokens: int = 0
    finished: bool = False
    required_blocks: int = 0
    last_logits: torch.Tensor | None = None
    prefill_offset: int = 0
    status: RequestStatus = RequestStatus.PENDING
    error: Exception | None = None
    _base: torch.Tensor | None = field(default=None, init=False, repr=False)
    _appended: list[int] = field(default_factory=list, init=False, repr=False)
    _cached: torch.Tensor | None = field(default=None, init=False, repr=False)

    def __post_init__(self) -> None:
        self._base = self.prompt

    @property
    def sequence(self) -> torch.Tensor:
        if not self._appended:
            return self._base
        if self._cached is None or self._cached.shape[1] != self._base.shape[1] + len(self._appended):
            tail = torch.tensor([self._appended], dtype=self._base.dtype, device=self._base.device)
            self._cached = torch.cat((self._base, tail), dim=1)
        return self._cached

    @sequence.setter
    def sequence(self, value: torch.Tensor) -> None:
        self._base = value
        self._appended = []
        self._cached = None

    def append_token(self, token_id: int) -> None:
        self._appended.append(int(token_id))
