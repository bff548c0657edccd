"""Prefill engine and continuous-batching decode engine in one process
(the reference's generation/pd_scheduler.py API).

Design: the decode side is an ordinary :class:`ContinuousBatchingScheduler`
over the decode pool (requests enter it already prefilled); this class keeps
only the FIFO of prompts that have not been prefilled and, around each decode
step, *refills* the decode batch from it through :class:`PDPair` hand-offs.

A refill takes the longest prefix of the FIFO the decode side can accept --
free batch slots, and worst-case decode blocks (prompt + new tokens - 1) not
yet reserved -- that the prefill pool can hold at once (and, with
``max_prefill_tokens_per_step``, within that many prompt tokens; the first
request always goes).  The whole prefix is prefilled in ONE ragged forward
and moved block to block into the decode pool.  The reference prefills and
hands over one request at a time (pd_scheduler.py:136-181); grouping changes
no result: the decode pool receives the requests in the same order, so block
tables, tokens and events are the same.  When a grouped hand-off fails, the
group is retried one request at a time, so only the request that cannot be
handed over fails and later requests proceed (the reference's semantics).

Step order, as in the reference (pd_scheduler.py:222-246): decode the running
batch, then refill; an empty decode side is refilled, decoded once and
refilled again within the same step.
"""

from __future__ import annotations

from collections import deque

import torch

from ..paged_cache import PagedKVCache
from .config import GenerationConfig
from .events import SchedulerStepOutput
from .pd_handoff import PDPair, blocks_for
from .request import PagedRequest, RequestStatus
from .scheduler import ContinuousBatchingScheduler


class PDContinuousBatchingScheduler:
    """Pipeline prefill on one device and continuous decode on another."""

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
        self.pair = PDPair.checked(prefill_model, decode_model, prefill_cache, decode_cache)
        self.config = config
        self.decode_scheduler = ContinuousBatchingScheduler(
            decode_model, config, decode_cache, max_batch_size, release_on_token_limit=True
        )
        self.pending_requests: deque[PagedRequest] = deque()
        self.completed_requests: list[PagedRequest] = []
        self._requests: dict[str, PagedRequest] = {}
        self._closed = False

    # ------------------------------------------------ the reference's attributes
    prefill_model = property(lambda self: self.pair.prefill_model)
    decode_model = property(lambda self: self.pair.decode_model)
    prefill_cache = property(lambda self: self.pair.prefill_cache)
    decode_cache = property(lambda self: self.pair.decode_cache)
    max_batch_size = property(lambda self: self.decode_scheduler.max_batch_size)
    block_budget = property(lambda self: self.decode_scheduler.block_budget)

    @property
    def has_work(self) -> bool:
        return bool(self.pending_requests) or self.decode_scheduler.has_work

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
        if sequence_id not in self._requests:
            raise KeyError(sequence_id)
        return self._requests[sequence_id]

    # -------------------------------------------------------------- submission
    def add_request(self, sequence_id: str, prompt: torch.Tensor) -> PagedRequest:
        """Queue a prompt (FIFO).  Rejects, in this order: a closed scheduler, a
        resubmitted id, a malformed prompt or an id already in either pool, a
        request longer than the decode model's max_seq_len, and one whose
        worst case exceeds the decode pool or whose prompt exceeds the prefill pool."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        if sequence_id in self._requests:
            raise ValueError(f"sequence ID already submitted: {sequence_id}")
        self.pair.check_new(sequence_id, prompt)
        length = prompt.shape[1]
        if length + self.config.max_new_tokens > self.decode_model.config.max_seq_len:
            raise ValueError(f"request exceeds max model length: {sequence_id}")
        worst_case = blocks_for(length + self.config.max_new_tokens - 1, self.decode_cache.block_size)
        if worst_case > self.block_budget:
            raise ValueError(f"request cannot fit in decode cache: {sequence_id}")
        if blocks_for(length, self.prefill_cache.block_size) > self.prefill_cache.allocator.num_blocks:
            raise ValueError(f"request cannot fit in prefill cache: {sequence_id}")
        request = PagedRequest(sequence_id=sequence_id, prompt=prompt, required_blocks=worst_case)
        self._requests[sequence_id] = request
        self.pending_requests.append(request)
        return request

    # ------------------------------------------------------------------ refill
    def _next_group(self) -> list[PagedRequest]:
        """The FIFO prefix the decode side accepts and the prefill pool holds."""
        slots = self.max_batch_size - self.active_count
        room = self.block_budget - self.decode_scheduler.reserved_blocks
        token_cap = self.config.max_prefill_tokens_per_step
        group: list[PagedRequest] = []
        tokens = 0
        for request in self.pending_requests:
            if len(group) == slots or request.required_blocks > room:
                break
            length = request.prompt.shape[1]
            if group and token_cap is not None and tokens + length > token_cap:
                break
            if group and not self.pair.prefill_fits([r.prompt for r in group] + [request.prompt]):
                break
            group.append(request)
            room -= request.required_blocks
            tokens += length
        return group

    def _admit(self, request: PagedRequest, last_logits: torch.Tensor) -> None:
        on_decode = request.prompt.to(self.pair.decode_device)
        request.prompt = on_decode
        request.sequence = on_decode
        self.decode_scheduler.add_prefilled_request(request, last_logits)

    def _fail(self, request: PagedRequest, error: Exception) -> PagedRequest:
        self.pair.forget(request.sequence_id)
        request.status = RequestStatus.FAILED
        request.error = error
        return request

    def _hand_over(self, group: list[PagedRequest]) -> list[PagedRequest]:
        """Hand the group over and admit it; returns the requests that failed."""
        try:
            logits = self.pair.hand_off([r.sequence_id for r in group], [r.prompt for r in group])
        except Exception as error:
            if len(group) == 1:
                return [self._fail(group[0], error)]
            # the grouped hand-off left nothing behind in either pool: retry the
            # requests alone so that only the one that cannot be handed over fails
            return [f for r in group for f in self._hand_over([r])]
        failed = []
        for request, row in zip(group, logits):
            try:
                self._admit(request, row)
            except Exception as error:
                failed.append(self._fail(request, error))
        return failed

    def _refill(self) -> list[PagedRequest]:
        failed: list[PagedRequest] = []
        while self.pending_requests:
            group = self._next_group()
            if not group:
                break
            for _ in group:
                self.pending_requests.popleft()
            failed.extend(self._hand_over(group))
        return failed

    # ----------------------------------------------------------------- control
    def cancel_request(self, sequence_id: str) -> bool:
        """Cancel a queued or decoding request and free its blocks."""
        request = self.get_request(sequence_id)
        if request.status is RequestStatus.ACTIVE:
            if not self.decode_scheduler.cancel_request(sequence_id):
                return False
        elif request.status is RequestStatus.PENDING:
            self.pending_requests = deque(r for r in self.pending_requests if r is not request)
            request.status = RequestStatus.CANCELLED
        else:
            return False
        self.completed_requests.append(request)
        return True

    def close(self) -> tuple[PagedRequest, ...]:
        """Cancel every unfinished request (queued first, then decoding) and free
        both pools; a second call returns ()."""
        if self._closed:
            return ()
        self._closed = True
        cancelled = list(self.pending_requests)
        self.pending_requests.clear()
        for request in cancelled:
            request.status = RequestStatus.CANCELLED
        cancelled.extend(self.decode_scheduler.close())
        for sequence_id in self._requests:
            self.pair.forget(sequence_id)
        self.completed_requests.extend(cancelled)
        return tuple(cancelled)

    def _decode_once(self, finished: list[PagedRequest]):
        out = self.decode_scheduler.step()
        finished.extend(out.terminal_requests)
        return out.token_events

    @torch.inference_mode()
    def step(self) -> SchedulerStepOutput:
        """Decode the running batch, then refill it from the queue (an empty decode
        side is refilled, decoded once and refilled again)."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        finished: list[PagedRequest] = []
        events = ()
        if self.active_count:
            events = self._decode_once(finished)
            finished.extend(self._refill())
        else:
            finished.extend(self._refill())
            if self.active_count:
                events = self._decode_once(finished)
                finished.extend(self._refill())
        self.completed_requests.extend(finished)
        return SchedulerStepOutput(events, tuple(finished))

    def run_until_idle(self) -> tuple[PagedRequest, ...]:
        """Step until every submitted request is terminal."""
        done: list[PagedRequest] = []
        while self.has_work:
            done.extend(self.step().terminal_requests)
        return tuple(done)
