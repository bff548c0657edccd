"""Prefill on one device, continuous decode on another (reference generation/pd_scheduler.py).

Same admission, handoff and cancellation semantics as the reference; the
handoff copies KV blocks prefill-pool -> decode-pool with one kernel
(:func:`transfer_sequence`, NVLink peer stores across GPUs).
"""

from __future__ import annotations

from collections import deque

import torch

from ..paged_cache import PagedKVCache, transfer_sequence
from .config import GenerationConfig
from .events import SchedulerStepOutput
from .paged_prefill import _validate_paged_prefill_inputs, paged_prefill
from .pd_greedy import _release_if_allocated, _validate_model_cache
from .request import PagedRequest, RequestStatus
from .scheduler import ContinuousBatchingScheduler


class PDContinuousBatchingScheduler:
    def __init__(
        self,
        prefill_model,
        decode_model,
        config: GenerationConfig,
        prefill_cache: PagedKVCache,
        decode_cache: PagedKVCache,
        max_batch_size: int,
    ) -> None:
        if not config.use_cache:
            raise ValueError("P/D scheduling requires config.use_cache=True")
        if prefill_cache is decode_cache:
            raise ValueError("prefill_cache and decode_cache must be different caches")
        _validate_model_cache(prefill_model, prefill_cache, "prefill")
        _validate_model_cache(decode_model, decode_cache, "decode")
        self.prefill_model = prefill_model
        self.decode_model = decode_model
        self.config = config
        self.prefill_cache = prefill_cache
        self.decode_cache = decode_cache
        self.decode_scheduler = ContinuousBatchingScheduler(
            decode_model, config, decode_cache, max_batch_size, release_on_token_limit=True
        )
        self.max_batch_size = self.decode_scheduler.max_batch_size
        self.block_budget = self.decode_scheduler.block_budget
        self.pending_requests: deque[PagedRequest] = deque()
        self.completed_requests: list[PagedRequest] = []
        self._requests: dict[str, PagedRequest] = {}
        self._closed = False

    @property
    def has_work(self) -> bool:
        return bool(self.pending_requests or self.decode_scheduler.has_work)

    @property
    def pending_count(self) -> int:
        return len(self.pending_requests)

    @property
    def active_count(self) -> int:
        return self.decode_scheduler.active_count

    @property
    def free_block_count(self) -> int:
        return self.decode_cache.allocator.free_block_count

    @property
    def is_closed(self) -> bool:
        return self._closed

    def get_request(self, sequence_id: str) -> PagedRequest:
        try:
            return self._requests[sequence_id]
        except KeyError:
            raise KeyError(sequence_id) from None

    def add_request(self, sequence_id: str, prompt: torch.Tensor) -> PagedRequest:
        """Reference pd_scheduler.py:198-251."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        if sequence_id in self._requests:
            raise ValueError(f"sequence ID already submitted: {sequence_id}")
        _validate_paged_prefill_inputs((prompt,), self.prefill_cache, (sequence_id,))
        if sequence_id in self.decode_cache._block_tables:
            raise ValueError(f"sequence ID already exists: {sequence_id}")
        if prompt.shape[1] + self.config.max_new_tokens > self.decode_model.config.max_seq_len:
            raise ValueError(f"request exceeds max model length: {sequence_id}")
        dbs = self.decode_cache.block_size
        required = (prompt.shape[1] + self.config.max_new_tokens - 1 + dbs - 1) // dbs
        if required > self.block_budget:
            raise ValueError(f"request cannot fit in decode cache: {sequence_id}")
        pbs = self.prefill_cache.block_size
        if (prompt.shape[1] + pbs - 1) // pbs > self.prefill_cache.allocator.num_blocks:
            raise ValueError(f"request cannot fit in prefill cache: {sequence_id}")
        request = PagedRequest(sequence_id=sequence_id, prompt=prompt, required_blocks=required)
        self.pending_requests.append(request)
        self._requests[sequence_id] = request
        return request

    def _handoff_request(self, request: PagedRequest) -> None:
        """Prefill, move KV to the decode pool, admit for decode (reference :253-274)."""
        device = self.decode_cache.keys.device
        try:
            logits = paged_prefill(self.prefill_model, (request.prompt,), self.prefill_cache, (request.sequence_id,))
            transfer_sequence(self.prefill_cache, self.decode_cache, request.sequence_id)
            decode_prompt = request.prompt.to(device)
            last_logits = logits[0].to(device)
            request.prompt = decode_prompt
            request.sequence = decode_prompt
            self.decode_scheduler.add_prefilled_request(request, last_logits)
        except Exception:
            _release_if_allocated(self.decode_cache, request.sequence_id)
            raise
        finally:
            _release_if_allocated(self.prefill_cache, request.sequence_id)

    def _admit_pending_requests(self) -> list[PagedRequest]:
        failed: list[PagedRequest] = []
        while self.pending_requests and self.active_count < self.max_batch_size:
            head = self.pending_requests[0]
            if self.decode_scheduler.reserved_blocks + head.required_blocks > self.block_budget:
                break
            self.pending_requests.popleft()
            try:
                self._handoff_request(head)
            except Exception as error:
                head.status = RequestStatus.FAILED
                head.error = error
                failed.append(head)
        return failed

    def cancel_request(self, sequence_id: str) -> bool:
        request = self.get_request(sequence_id)
        if request.status is RequestStatus.PENDING:
            self.pending_requests = deque(r for r in self.pending_requests if r is not request)
            request.status = RequestStatus.CANCELLED
            self.completed_requests.append(request)
            return True
        if request.status is RequestStatus.ACTIVE:
            cancelled = self.decode_scheduler.cancel_request(sequence_id)
            if cancelled:
                self.completed_requests.append(request)
            return cancelled
        return False

    def close(self) -> tuple[PagedRequest, ...]:
        if self._closed:
            return ()
        self._closed = True
        cancelled: list[PagedRequest] = []
        for request in self.pending_requests:
            request.status = RequestStatus.CANCELLED
            cancelled.append(request)
        self.pending_requests.clear()
        cancelled.extend(self.decode_scheduler.close())
        for request in self._requests.values():
            _release_if_allocated(self.prefill_cache, request.sequence_id)
            _release_if_allocated(self.decode_cache, request.sequence_id)
        self.completed_requests.extend(cancelled)
        return tuple(cancelled)

    @torch.inference_mode()
    def step(self) -> SchedulerStepOutput:
        """Decode first, then fill free decode slots through prefill (reference :339-363)."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        events = ()
        completed_now: list[PagedRequest] = []
        had_batch = self.active_count > 0
        if had_batch:
            out = self.decode_scheduler.step()
            events = out.token_events
            completed_now.extend(out.terminal_requests)
        completed_now.extend(self._admit_pending_requests())
        if not had_batch and self.active_count > 0:
            out = self.decode_scheduler.step()
            events = out.token_events
            completed_now.extend(out.terminal_requests)
            completed_now.extend(self._admit_pending_requests())
        self.completed_requests.extend(completed_now)
        return SchedulerStepOutput(events, tuple(completed_now))

    def run_until_idle(self) -> tuple[PagedRequest, ...]:
        completed = []
        while self.has_work:
            completed.extend(self.step().terminal_requests)
        return tuple(completed)
