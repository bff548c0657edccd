"""Continuous-batching scheduler (reference generation/scheduler.py:17-585).

The step plan is the reference's, decision for decision: FIFO admission
against a worst-case block reservation, chunked prefill under a round-robin
token budget, and a unified ragged call whose order is *prefill chunks
first, then one decode token per surviving request*.  Those orders decide
the allocation order inside ``forward_ragged`` and therefore the block
tables, which must be bit-identical.

Host-side differences that do not change any result:

* EOS checks use the token ids already copied to the host for the token
  events instead of one device read per request;
* generated tokens are appended to a host list (``PagedRequest.sequence``
  materialises lazily) instead of one device ``cat`` per request per step.
"""

from __future__ import annotations

from collections import deque

import torch

from .. import ops
from ..paged_cache import PagedKVCache
from .config import GenerationConfig
from .events import SchedulerStepOutput, TokenEvent
from .paged_prefill import _validate_paged_prefill_inputs, paged_prefill, paged_prefill_chunks
from .request import PagedRequest, RequestStatus


def _rows_view(rows: list[torch.Tensor]) -> torch.Tensor | None:
    """``rows`` as one [len, V] tensor without a copy when they are consecutive
    rows of one buffer (the decode batch's logits), else None."""
    first = rows[0]
    if first.ndim != 1 or first.stride(0) != 1:
        return None
    n = first.shape[0]
    step = n * first.element_size()
    p0 = first.data_ptr()
    storage = first.untyped_storage().data_ptr()
    for i, r in enumerate(rows):
        if (r.ndim != 1 or r.shape[0] != n or r.dtype != first.dtype or r.stride(0) != 1
                or r.data_ptr() != p0 + i * step or r.untyped_storage().data_ptr() != storage):
            return None
    return first.as_strided((len(rows), n), (n, 1))


class _PendingTokens:
    """Sampled token ids on their way to the host: a pinned buffer filled by an
    asynchronous copy, and the event that marks the copy's completion."""

    def __init__(self, tokens: torch.Tensor) -> None:
        flat = tokens.reshape(-1)
        self.host = torch.empty(flat.shape, dtype=flat.dtype, pin_memory=True)
        self.host.copy_(flat, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(flat.device))

    def values(self) -> list[int]:
        self.event.synchronize()
        return self.host.tolist()


class ContinuousBatchingScheduler:
    """Schedule dynamically submitted requests over one shared paged cache."""

    def __init__(
        self,
        model,
        config: GenerationConfig,
        paged_cache: PagedKVCache,
        max_batch_size: int,
        *,
        release_on_token_limit: bool = True,
    ) -> None:
        if not config.use_cache:
            raise ValueError("continuous batching requires config.use_cache=True")
        if isinstance(max_batch_size, bool) or not isinstance(max_batch_size, int) or max_batch_size <= 0:
            raise ValueError("max_batch_size must be a positive integer")
        if not isinstance(paged_cache, PagedKVCache):
            raise TypeError("paged_cache must be a PagedKVCache")
        self.model = model
        self.config = config
        self.paged_cache = paged_cache
        self.max_batch_size = max_batch_size
        self.release_on_token_limit = release_on_token_limit
        self.block_budget = paged_cache.allocator.free_block_count
        self.pending_requests: deque[PagedRequest] = deque()
        self.prefilling_requests: list[PagedRequest] = []
        self.active_requests: list[PagedRequest] = []
        self.completed_requests: list[PagedRequest] = []
        self.reserved_blocks = 0
        self._requests: dict[str, PagedRequest] = {}
        self._closed = False

    # ---------------------------------------------------------- inspection
    @property
    def has_work(self) -> bool:
        return bool(self.pending_requests or self.prefilling_requests or self.active_requests)

    @property
    def pending_count(self) -> int:
        return len(self.pending_requests)

    @property
    def active_count(self) -> int:
        return len(self.active_requests)

    @property
    def prefilling_count(self) -> int:
        return len(self.prefilling_requests)

    @property
    def free_block_count(self) -> int:
        return self.paged_cache.allocator.free_block_count

    @property
    def is_closed(self) -> bool:
        return self._closed

    def get_request(self, sequence_id: str) -> PagedRequest:
        try:
            return self._requests[sequence_id]
        except KeyError:
            raise KeyError(sequence_id) from None

    # ----------------------------------------------------------- admission
    def _required_blocks(self, prompt_length: int) -> int:
        # Worst case: prompt plus every generated token except the last,
        # which is never written (reference scheduler.py:109-115).
        bs = self.paged_cache.block_size
        return (prompt_length + self.config.max_new_tokens - 1 + bs - 1) // bs

    def add_request(self, sequence_id: str, prompt: torch.Tensor) -> PagedRequest:
        """Queue a prompt FIFO (reference scheduler.py:89-128)."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        if sequence_id in self._requests:
            raise ValueError(f"sequence ID already submitted: {sequence_id}")
        _validate_paged_prefill_inputs((prompt,), self.paged_cache, (sequence_id,))
        max_len = getattr(getattr(self.model, "config", None), "max_seq_len", None)
        if max_len is not None and prompt.shape[1] + self.config.max_new_tokens > max_len:
            raise ValueError(f"request exceeds max model length: {sequence_id}")
        required = self._required_blocks(prompt.shape[1])
        if required > self.block_budget:
            raise ValueError(f"request cannot fit in paged cache: {sequence_id}")
        request = PagedRequest(sequence_id=sequence_id, prompt=prompt, required_blocks=required)
        self.pending_requests.append(request)
        self._requests[sequence_id] = request
        return request

    def add_prefilled_request(self, request: PagedRequest, last_logits: torch.Tensor) -> None:
        """Admit a request whose KV is already in this cache (reference scheduler.py:130-181)."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        if not isinstance(request, PagedRequest):
            raise TypeError("request must be a PagedRequest")
        if request.sequence_id in self._requests:
            raise ValueError(f"sequence ID already submitted: {request.sequence_id}")
        if request.status is not RequestStatus.PENDING:
            raise ValueError("prefilled request must have pending status")
        rb = request.required_blocks
        if isinstance(rb, bool) or not isinstance(rb, int) or rb <= 0:
            raise ValueError("prefilled request must reserve at least one block")
        if len(self.active_requests) >= self.max_batch_size:
            raise ValueError("decode batch is full")
        device = self.paged_cache.keys.device
        if request.prompt.device != device:
            raise ValueError("prefilled prompt must be on the decode cache device")
        if not isinstance(last_logits, torch.Tensor):
            raise TypeError("last_logits must be a torch.Tensor")
        if last_logits.ndim != 1:
            raise ValueError("last_logits must be a 1D tensor")
        if last_logits.device != device:
            raise ValueError("last_logits must be on the decode cache device")
        if self.reserved_blocks + rb > self.block_budget:
            raise ValueError("not enough reserved decode cache blocks")
        if request.sequence_id not in self.paged_cache._block_tables:
            raise ValueError("prefilled request is missing decode KV")
        if self.paged_cache.get_sequence_length(request.sequence_id) != request.prompt.shape[1]:
            raise ValueError("decode KV length must match the prompt length")
        request.last_logits = last_logits
        request.status = RequestStatus.ACTIVE
        self.active_requests.append(request)
        self.reserved_blocks += rb
        self._requests[request.sequence_id] = request

    def _release_request_cache(self, sequence_id: str) -> None:
        if sequence_id in self.paged_cache._block_tables:
            self.paged_cache.release(sequence_id)

    def _admit_pending_requests(self) -> list[PagedRequest]:
        """Non-chunked admission with one batched prefill (reference scheduler.py:190-253)."""
        if self.config.prefill_chunk_size is not None:
            self._admit_chunked_requests()
            return []
        failed: list[PagedRequest] = []
        admitted: list[PagedRequest] = []
        while self.pending_requests and len(self.active_requests) + len(admitted) < self.max_batch_size:
            head = self.pending_requests[0]
            pending_blocks = sum(r.required_blocks for r in admitted)
            if self.reserved_blocks + pending_blocks + head.required_blocks > self.block_budget:
                break
            admitted.append(self.pending_requests.popleft())
        if not admitted:
            return failed
        try:
            logits = paged_prefill(
                self.model,
                tuple(r.prompt for r in admitted),
                self.paged_cache,
                tuple(r.sequence_id for r in admitted),
            )
        except Exception:
            # One bad prompt must not fail its batch mates: retry one by one.
            for request in admitted:
                try:
                    single = paged_prefill(self.model, (request.prompt,), self.paged_cache, (request.sequence_id,))
                    request.last_logits = single[0]
                except Exception as error:
                    self._release_request_cache(request.sequence_id)
                    request.status = RequestStatus.FAILED
                    request.error = error
                    failed.append(request)
                    continue
                request.status = RequestStatus.ACTIVE
                self.active_requests.append(request)
                self.reserved_blocks += request.required_blocks
            return failed
        for request, row in zip(admitted, logits):
            request.last_logits = row
            request.status = RequestStatus.ACTIVE
            self.active_requests.append(request)
            self.reserved_blocks += request.required_blocks
        return failed

    def _admit_chunked_requests(self) -> None:
        """Reference scheduler.py:255-265."""
        occupied = len(self.active_requests) + len(self.prefilling_requests)
        while self.pending_requests and occupied < self.max_batch_size:
            head = self.pending_requests[0]
            if self.reserved_blocks + head.required_blocks > self.block_budget:
                break
            self.pending_requests.popleft()
            head.status = RequestStatus.PREFILLING
            self.prefilling_requests.append(head)
            self.reserved_blocks += head.required_blocks
            occupied += 1

    def _take_prefill_chunks(self) -> tuple[list[PagedRequest], tuple[torch.Tensor, ...]]:
        """Round-robin chunks under the step's token budget (reference scheduler.py:267-298)."""
        chunk = self.config.prefill_chunk_size
        assert chunk is not None
        budget = self.config.max_prefill_tokens_per_step
        if budget is None:
            budget = sum(min(chunk, r.prompt.shape[1] - r.prefill_offset) for r in self.prefilling_requests)
        taken: list[PagedRequest] = []
        pieces: list[torch.Tensor] = []
        while self.prefilling_requests and budget > 0:
            request = self.prefilling_requests.pop(0)
            count = min(chunk, request.prompt.shape[1] - request.prefill_offset, budget)
            pieces.append(request.prompt[:, request.prefill_offset : request.prefill_offset + count])
            taken.append(request)
            budget -= count
        return taken, tuple(pieces)

    def _finish_prefill_chunks(
        self,
        requests: list[PagedRequest],
        chunks: tuple[torch.Tensor, ...],
        logits: torch.Tensor,
    ) -> None:
        """Reference scheduler.py:300-315: finished prompts go active, others requeue last."""
        for request, row, piece in zip(requests, logits, chunks):
            request.prefill_offset += piece.shape[1]
            request.last_logits = row
            if request.prefill_offset == request.prompt.shape[1]:
                request.status = RequestStatus.ACTIVE
                self.active_requests.append(request)
            else:
                self.prefilling_requests.append(request)

    # ---------------------------------------------------------- lifecycle
    def cancel_request(self, sequence_id: str) -> bool:
        """Reference scheduler.py:317-354."""
        request = self._requests.get(sequence_id)
        if request is None:
            raise KeyError(sequence_id)
        if request.status not in (RequestStatus.PENDING, RequestStatus.PREFILLING, RequestStatus.ACTIVE):
            return False
        if request.status is RequestStatus.PENDING:
            self.pending_requests = deque(r for r in self.pending_requests if r is not request)
        elif request.status is RequestStatus.PREFILLING:
            self.prefilling_requests = [r for r in self.prefilling_requests if r is not request]
            self.reserved_blocks -= request.required_blocks
            self._release_request_cache(request.sequence_id)
        else:
            self.active_requests = [r for r in self.active_requests if r is not request]
            self.reserved_blocks -= request.required_blocks
            self._release_request_cache(request.sequence_id)
        request.status = RequestStatus.CANCELLED
        self.completed_requests.append(request)
        return True

    def close(self) -> tuple[PagedRequest, ...]:
        """Cancel everything unfinished and release all cache (reference scheduler.py:356-379)."""
        if self._closed:
            return ()
        self._closed = True
        cancelled: list[PagedRequest] = []
        for request in (*self.pending_requests, *self.prefilling_requests, *self.active_requests):
            request.status = RequestStatus.CANCELLED
            cancelled.append(request)
        for request in self._requests.values():
            self._release_request_cache(request.sequence_id)
        self.pending_requests.clear()
        self.prefilling_requests.clear()
        self.active_requests.clear()
        self.reserved_blocks = 0
        self.completed_requests.extend(cancelled)
        return tuple(cancelled)

    # --------------------------------------------------------------- steps
    def _sample(
        self, requests: list[PagedRequest], *, defer: bool = False
    ) -> tuple[torch.Tensor, list[int] | _PendingTokens]:
        """Greedy next tokens on the device, and their values for the host.

        ``defer`` (CUDA only) starts the copy to the host without waiting for
        it: the caller can queue the next forward first and read the values
        (``_PendingTokens.values``) while the GPU runs it.
        """
        rows = []
        for request in requests:
            if request.last_logits is None:
                raise RuntimeError("active request is missing logits")
            rows.append(request.last_logits)
        if not rows:
            empty = torch.empty((0, 1), dtype=torch.long, device=self.paged_cache.keys.device)
            return empty, []
        stacked = _rows_view(rows)
        if stacked is None:
            stacked = torch.stack(rows)
        if stacked.is_cuda and stacked.ndim == 2 and len(rows) <= ops.ARGMAX_MAX_ROWS:
            next_tokens = ops.argmax_rows(stacked).unsqueeze(-1)  # one launch, torch.argmax's answer
        else:
            next_tokens = stacked.argmax(dim=-1, keepdim=True)
        if defer and next_tokens.is_cuda:
            return next_tokens, _PendingTokens(next_tokens)
        return next_tokens, next_tokens.squeeze(-1).tolist()

    def _retire(
        self,
        requests: list[PagedRequest],
        token_ids: list[int] | None,
        completed_now: list[PagedRequest],
    ) -> list[int]:
        """Append sampled tokens; retire on EOS / token limit; return survivor indices.

        ``token_ids`` None (no EOS configured, so only the token count decides)
        leaves the appends to the caller, once the values have reached the host.
        """
        eos = self.config.eos_token_id
        if token_ids is None and eos is not None:
            raise ValueError("token values are needed to check for the EOS token")
        survivors: list[int] = []
        for index, request in enumerate(requests):
            request.generated_tokens += 1
            if token_ids is not None:
                request.append_token(token_ids[index])
        for index, request in enumerate(requests):
            stopped = eos is not None and token_ids[index] == eos
            at_limit = request.generated_tokens >= self.config.max_new_tokens
            if stopped or at_limit:
                request.finished = stopped
                request.status = RequestStatus.COMPLETED
                self.reserved_blocks -= request.required_blocks
                if stopped or self.release_on_token_limit:
                    self._release_request_cache(request.sequence_id)
                completed_now.append(request)
            else:
                survivors.append(index)
        return survivors

    def _fail(self, requests: list[PagedRequest], error: Exception, completed_now: list[PagedRequest]) -> None:
        for request in requests:
            request.status = RequestStatus.FAILED
            request.error = error
            self.reserved_blocks -= request.required_blocks
            self._release_request_cache(request.sequence_id)
            completed_now.append(request)

    def _step_unified_ragged(self) -> SchedulerStepOutput:
        """Chunked prefill and decode in one flattened call (reference scheduler.py:381-483)."""
        self._admit_chunked_requests()
        if not self.active_requests and not self.prefilling_requests and self.pending_requests:
            raise RuntimeError("pending requests cannot be admitted")
        completed_now: list[PagedRequest] = []
        decoding = list(self.active_requests)
        # Without an EOS token the schedule depends on token counts only, so the
        # next forward is queued before the sampled values are read back: the
        # host bookkeeping of this step then overlaps the GPU's next step.
        next_tokens, sampled = self._sample(decoding, defer=self.config.eos_token_id is None)
        token_ids = None if isinstance(sampled, _PendingTokens) else sampled
        keep = self._retire(decoding, token_ids, completed_now)
        survivors = [decoding[i] for i in keep]
        survivor_tokens = [next_tokens[i : i + 1] for i in keep]
        self.active_requests = survivors

        prefill_requests, prefill_chunks = self._take_prefill_chunks()
        ragged = [*prefill_requests, *survivors]
        if ragged:
            try:
                logits = paged_prefill_chunks(
                    self.model,
                    (*prefill_chunks, *survivor_tokens),
                    self.paged_cache,
                    tuple(r.sequence_id for r in ragged),
                )
            except Exception as error:
                self._fail(ragged, error, completed_now)
                self.active_requests = []
            else:
                n = len(prefill_requests)
                self._finish_prefill_chunks(prefill_requests, prefill_chunks, logits[:n])
                for request, row in zip(survivors, logits[n:]):
                    request.last_logits = row
        if token_ids is None:
            token_ids = sampled.values()
            for request, token in zip(decoding, token_ids):
                request.append_token(token)
        events = tuple(TokenEvent(r.sequence_id, token_ids[i]) for i, r in enumerate(decoding))
        self.completed_requests.extend(completed_now)
        return SchedulerStepOutput(events, tuple(completed_now))

    @torch.inference_mode()
    def step(self) -> SchedulerStepOutput:
        """One iteration (reference scheduler.py:486-578)."""
        if self._closed:
            raise RuntimeError("scheduler is closed")
        if self.config.prefill_chunk_size is not None:
            return self._step_unified_ragged()
        completed_now = self._admit_pending_requests()
        if not self.active_requests:
            if self.pending_requests and not self.prefilling_requests:
                raise RuntimeError("pending requests cannot be admitted")
            self.completed_requests.extend(completed_now)
            return SchedulerStepOutput((), tuple(completed_now))
        decoding = list(self.active_requests)
        # as in _step_unified_ragged: without an EOS token the next forward is
        # queued before the sampled values are read back
        next_tokens, sampled = self._sample(decoding, defer=self.config.eos_token_id is None)
        token_ids = None if isinstance(sampled, _PendingTokens) else sampled
        keep = self._retire(decoding, token_ids, completed_now)
        survivors = [decoding[i] for i in keep]
        self.active_requests = survivors
        if survivors:
            try:
                logits = self.model(
                    next_tokens[keep],
                    kv_cache=self.paged_cache,
                    sequence_ids=tuple(r.sequence_id for r in survivors),
                )
                for i, request in enumerate(survivors):
                    request.last_logits = logits[i, -1]
            except Exception as error:
                self._fail(survivors, error, completed_now)
                self.active_requests = []
        if token_ids is None:
            token_ids = sampled.values()
            for request, token in zip(decoding, token_ids):
                request.append_token(token)
        events = tuple(TokenEvent(sequence_id=r.sequence_id, token_id=token_ids[i]) for i, r in enumerate(decoding))
        completed_now.extend(self._admit_pending_requests())
        self.completed_requests.extend(completed_now)
        return SchedulerStepOutput(events, tuple(completed_now))

    def run_until_idle(self) -> tuple[PagedRequest, ...]:
        completed: list[PagedRequest] = []
        while self.has_work:
            completed.extend(self.step().terminal_requests)
        return tuple(completed)
