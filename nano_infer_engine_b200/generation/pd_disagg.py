"""Prefill/decode disaggregation with one process per GPU.

The reference runs P/D inside one process that owns two devices
(generation/pd_scheduler.py:136-181, service/runtime.py:277-358): prefill,
``export_sequence`` on the prefill device, ``import_sequence`` with a
per-block cross-device ``copy_`` on the decode device, then
``add_prefilled_request``.  Here each GPU has its own process:

* a **pair** is (prefill rank, decode rank); a deterministic router assigns
  requests to pairs (least outstanding work);
* at set-up the prefill rank exports its KV pool with CUDA IPC and the
  decode rank maps it on its own device (``ops.ipc_import``);
* the prefill rank prefills batches of prompts as one ragged call, reads the
  greedy first tokens, and sends a HANDOFF message per request with its
  length, first token and physical block ids;
* the decode rank allocates blocks in its pool, **pulls** the blocks over
  NVLink with the block-copy kernel (zeroed tail as in the reference export),
  admits the request into its own continuous-batching scheduler and, once the
  copy has completed, sends an ACK so the prefill rank can free its blocks.

Messages are int64 records in the process group's key-value store, polled
without blocking.  The GPU-specific steps (prefill, block import) are
injectable so the protocol runs with gloo on CPU in tests.
"""

from __future__ import annotations

import pickle
import time
from collections import deque
from collections.abc import Callable
from dataclasses import dataclass

import numpy as np
import torch

from .. import ops
from ..paged_cache import PagedKVCache
from .config import GenerationConfig
from .paged_prefill import paged_prefill_chunks
from .request import PagedRequest
from .scheduler import ContinuousBatchingScheduler

HANDOFF = 1
ACK = 2
DONE = 3
HEADER_WORDS = 8


def assign_groups(work: list[int], groups: int, decode_per_group: int) -> list[list[list[int]]]:
    """Request indices per group and per decode rank of the group: the router
    (``assign_pairs`` over the groups) picks the group, and inside it the same
    least-outstanding-work rule picks the decode rank the prefill rank hands
    the request to.  ``[group][decode slot] -> request indices``."""
    out = []
    for members in assign_pairs(work, groups):
        slots = assign_pairs([work[i] for i in members], decode_per_group)
        out.append([[members[j] for j in slot] for slot in slots])
    return out


def assign_pairs(work: list[int], num_pairs: int) -> list[list[int]]:
    """Request indices per pair: each request (in arrival order) goes to the pair
    with the least outstanding work so far (ties: lowest pair index)."""
    load = [0] * num_pairs
    out: list[list[int]] = [[] for _ in range(num_pairs)]
    for index, w in enumerate(work):
        pair = min(range(num_pairs), key=lambda p: (load[p], p))
        out[pair].append(index)
        load[pair] += w
    return out


class PairChannel:
    """Ordered int64 messages between the two ranks of a pair, polled without blocking.

    Messages travel through the process group's key-value store (any c10d
    ``Store``): the n-th message from rank a to rank b is key ``pd/a->b/n``,
    deleted by the receiver once read.  ``Store.check`` does not block, so
    both loops keep stepping their models while no message is waiting.
    """

    def __init__(self, store, me: int, peer: int, words: int) -> None:
        self.store = store
        self.words = words
        self._out = f"pd/{me}->{peer}/"
        self._in = f"pd/{peer}->{me}/"
        self._sent = 0
        self._received = 0

    def send(self, values: list[int]) -> None:
        if len(values) > self.words:
            raise ValueError("message longer than the channel's fixed size")
        msg = np.zeros(self.words, dtype=np.int64)
        msg[: len(values)] = values
        self.store.set(self._out + str(self._sent), msg.tobytes())
        self._sent += 1

    def poll(self, stop_after: int | None = None) -> list[list[int]]:
        """Every waiting message in order; with ``stop_after``, none past the first
        message of that type (later ones stay queued, e.g. the next pass's)."""
        out = []
        while True:
            key = self._in + str(self._received)
            if not self.store.check([key]):
                return out
            out.append(np.frombuffer(self.store.get(key), dtype=np.int64).tolist())
            self.store.delete_key(key)
            self._received += 1
            if stop_after is not None and out[-1][0] == stop_after:
                return out

    def close(self) -> None:
        """Messages are delivered when ``send`` returns; nothing is left in flight."""


class PipeChannel:
    """The same ordered int64 messages as :class:`PairChannel`, over two named
    pipes (one per direction) between the ranks of a pair on one node.

    A poll is one non-blocking ``read`` (no round trip to the store's server).
    Each pipe has one writer, so the byte stream keeps the records in order
    even when a write is partial; bytes the pipe cannot take yet wait in a
    local queue that every ``send`` and ``poll`` retries (neither side ever
    blocks on a full pipe, so the pair cannot deadlock).  Set-up: the lower
    rank of the pair creates the pipes in a fresh temporary directory and
    publishes its path in the store; both ends open non-blocking.
    """

    def __init__(self, store, me: int, peer: int, words: int, *, timeout_s: float = 60.0) -> None:
        import os
        import tempfile

        self.words = words
        self.bytes = 8 * words
        key = f"pd/pipe/{min(me, peer)}-{max(me, peer)}"
        if me < peer:
            self._dir = tempfile.mkdtemp(prefix="nie_pd_")
            for a, b in ((me, peer), (peer, me)):
                os.mkfifo(os.path.join(self._dir, f"{a}to{b}"))
            store.set(key, self._dir.encode())
        else:
            store.wait([key])
            self._dir = store.get(key).decode()
        self._os = os
        # open the read end first, non-blocking: opening a write end without a
        # reader fails with ENXIO, so retry it (bounded) until the peer's read end exists
        self._rfd = os.open(os.path.join(self._dir, f"{peer}to{me}"), os.O_RDONLY | os.O_NONBLOCK)
        wpath = os.path.join(self._dir, f"{me}to{peer}")
        deadline = time.monotonic() + timeout_s
        while True:
            try:
                self._wfd = os.open(wpath, os.O_WRONLY | os.O_NONBLOCK)
                break
            except OSError:
                if time.monotonic() > deadline:
                    raise TimeoutError(f"pair channel: peer {peer} never opened its end")
                time.sleep(0.001)
        self._owner = me < peer
        self._pending: deque[bytes] = deque()
        self._buf = b""

    def _flush(self) -> None:
        while self._pending:
            try:
                n = self._os.write(self._wfd, self._pending[0])
            except BlockingIOError:
                return
            if n < len(self._pending[0]):
                self._pending[0] = self._pending[0][n:]  # the rest follows in stream order
                return
            self._pending.popleft()

    def send(self, values: list[int]) -> None:
        if len(values) > self.words:
            raise ValueError("message longer than the channel's fixed size")
        msg = np.zeros(self.words, dtype=np.int64)
        msg[: len(values)] = values
        self._pending.append(msg.tobytes())
        self._flush()

    def poll(self, stop_after: int | None = None) -> list[list[int]]:
        """Every waiting message in order; with ``stop_after``, none past the first
        message of that type (later ones stay buffered, e.g. the next pass's)."""
        self._flush()
        while True:
            try:
                chunk = self._os.read(self._rfd, 1 << 16)
            except BlockingIOError:
                break
            if not chunk:
                break
            self._buf += chunk
        out = []
        while len(self._buf) >= self.bytes:
            out.append(np.frombuffer(self._buf[: self.bytes], dtype=np.int64).tolist())
            self._buf = self._buf[self.bytes:]
            if stop_after is not None and out[-1][0] == stop_after:
                break
        return out

    def close(self) -> None:
        """Deliver whatever is still queued (bounded), then release the pipes."""
        deadline = time.monotonic() + 60.0
        while self._pending and time.monotonic() < deadline:
            self._flush()
            if self._pending:
                time.sleep(0.0005)
        if self._pending:
            raise TimeoutError("pair channel: the peer stopped reading")

    def release(self) -> None:
        """Close both descriptors; the creating rank removes the pipes."""
        import shutil

        for fd in (self._rfd, self._wfd):
            try:
                self._os.close(fd)
            except OSError:
                pass
        if self._owner:
            shutil.rmtree(self._dir, ignore_errors=True)


@dataclass
class RemotePool:
    """The prefill rank's KV pool as mapped into the decode process."""

    keys_ptr: int
    values_ptr: int
    num_blocks: int
    bases: tuple[int, int]
    device: torch.device

    def close(self) -> None:
        for base in self.bases:
            ops.ipc_close(base, self.device)


def export_pool(cache: PagedKVCache) -> dict:
    kh, ko = ops.ipc_export(cache.keys)
    vh, vo = ops.ipc_export(cache.values)
    return {
        "keys": (kh, ko),
        "values": (vh, vo),
        "shape": tuple(cache.keys.shape),
        "dtype": str(cache.keys.dtype),
    }


def import_pool(exported: dict, cache: PagedKVCache) -> RemotePool:
    if tuple(exported["shape"][0:1] + exported["shape"][2:]) != (cache.num_layers, cache.block_size,
                                                                  cache.kv_head_num, cache.head_dim):
        raise ValueError("prefill and decode pools must share layers, block size and head geometry")
    if exported["dtype"] != str(cache.keys.dtype):
        raise ValueError("prefill and decode pools must share a dtype")
    kp, kb = ops.ipc_import(*exported["keys"], cache.device)
    vp, vb = ops.ipc_import(*exported["values"], cache.device)
    return RemotePool(kp, vp, exported["shape"][1], (kb, vb), cache.device)


def publish_pool(store, rank: int, cache: PagedKVCache) -> None:
    """Prefill rank: put its pool's IPC handles in the store for its decode peer."""
    store.set(f"pd/pool/{rank}", pickle.dumps(export_pool(cache)))


def open_peer_pool(store, peer: int, cache: PagedKVCache) -> RemotePool:
    """Decode rank: map the prefill peer's published pool onto ``cache``'s device."""
    key = f"pd/pool/{peer}"
    store.wait([key])
    return import_pool(pickle.loads(store.get(key)), cache)


def close_peer_pool(store, rank: int, remote: RemotePool) -> None:
    """Decode rank: unmap the peer pool and tell the exporter it may free it."""
    remote.close()
    store.set(f"pd/unmapped/{rank}", b"1")


def wait_pool_unmapped(store, peer: int) -> None:
    """Prefill rank: block until the decode peer has unmapped this rank's pool."""
    store.wait([f"pd/unmapped/{peer}"])


def gpu_import(remote: RemotePool, transfer_log: list | None = None):
    """Block import for the decode worker: allocate, pull over NVLink, advance.

    With ``transfer_log``, each pull appends ``(bytes moved, start event, end
    event)`` (timing events on the decode stream around the copy kernel).
    """

    def _import(cache: PagedKVCache, sequence_id: str, length: int, src_blocks: list[int]):
        n = -(-length // cache.block_size)
        cache.ensure_capacity(sequence_id, length)
        dst = cache.get_block_table(sequence_id)[:n]
        dev = cache.device
        stream = torch.cuda.current_stream(dev)
        src_t = torch.tensor(src_blocks[:n], dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        dst_t = torch.tensor(dst, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        if transfer_log is not None:
            begin = torch.cuda.Event(enable_timing=True)
            begin.record(stream)
        ops.copy_blocks_from_pointers(remote.keys_ptr, remote.values_ptr, remote.num_blocks, src_t, cache.keys,
                                      cache.values, dst_t, n, length % cache.block_size)
        cache.advance(sequence_id, length)
        event = torch.cuda.Event(enable_timing=transfer_log is not None)
        event.record(stream)
        if transfer_log is not None:
            moved = 2 * n * cache.num_layers * cache.block_size * cache.kv_head_num * cache.head_dim
            transfer_log.append((moved * cache.keys.element_size(), begin, event))
        return event

    return _import


@dataclass
class PrefillStats:
    requests: int = 0
    tokens: int = 0
    batches: int = 0


def run_prefill(
    model,
    cache: PagedKVCache,
    channel,
    requests: list[tuple[int, torch.Tensor]],
    *,
    token_budget: int = 8192,
    chunk_size: int | None = None,
    route: list[int] | None = None,
    arrival: list[float] | None = None,
    clock: Callable[[], float] = time.perf_counter,
    idle_sleep: float = 0.0,
    first_token_at: dict[int, float] | None = None,
) -> PrefillStats:
    """Prefill ``(index, prompt[1, n])`` requests in order and hand them to the decode peer.

    Batches are formed from arrived requests up to ``token_budget`` prompt
    tokens and the free blocks of ``cache``; a request's blocks are held
    until the decode peer acknowledges its copy.  With ``chunk_size`` a
    prompt is prefilled in chunks of at most that many tokens: each batch
    first continues the requests already started (oldest first), then starts
    arrived ones, the last chunk of a batch cut to fit the budget, so a long
    prompt shares its batches with the prompts behind it; a request is handed
    off after its last chunk (the reference prefills each prompt whole,
    generation/pd_scheduler.py:136-145).  Without it every prompt is one
    chunk and a batch never splits one.  ``channel`` is the decode peer's
    channel, or a list of channels when this rank feeds several decode ranks;
    ``route[k]`` then names the channel of request k.  Acknowledgements are
    taken from every channel and each one gets DONE.  ``arrival`` (``clock()`` times, same
    order as ``requests``) gates admission for open-loop runs;
    ``first_token_at`` receives, per request index, the ``clock()`` time at
    which its first token was known, so TTFT = first_token_at - arrival on one
    time base.
    """
    if chunk_size is not None and chunk_size <= 0:
        raise ValueError("chunk_size must be positive")
    channels = list(channel) if isinstance(channel, (list, tuple)) else [channel]
    if route is None:
        if len(channels) != 1:
            raise ValueError("route is required with several channels")
        route = [0] * len(requests)
    if len(route) != len(requests) or any(not 0 <= c < len(channels) for c in route):
        raise ValueError("route must name one channel per request")
    sent = [0] * len(channels)
    stats = PrefillStats()
    pending = deque(range(len(requests)))
    started: deque[int] = deque()  # chunked requests with prompt tokens still to prefill
    done: dict[int, int] = {}  # prompt tokens already in the cache, per started request
    held: dict[int, str] = {}
    bs = cache.block_size
    while pending or started or held:
        for ch in channels:
            for msg in ch.poll():
                if msg[0] == ACK:
                    cache.release(held.pop(msg[1]))
        batch: list[tuple[int, int, int]] = []  # (request, first token, end token) of each chunk
        tokens = 0
        # blocks not yet allocated and not promised to a started request: a
        # request starts only when its whole prompt fits, so started requests
        # always finish (their blocks are freed on the peer's ACK)
        free = cache.allocator.free_block_count
        free -= sum(-(-requests[k][1].shape[1] // bs) - (-(-done[k] // bs)) for k in started)
        for k in started:
            n, at = requests[k][1].shape[1], done[k]
            take = min(n - at, chunk_size, token_budget - tokens)
            if take <= 0:
                break
            batch.append((k, at, at + take))
            tokens += take
        now = clock()
        while pending and len(batch) == len(started) and tokens < token_budget:
            k = pending[0]
            if arrival is not None and arrival[k] > now:
                break
            n = requests[k][1].shape[1]
            take = n if chunk_size is None else min(n, chunk_size, token_budget - tokens)
            if chunk_size is None and batch and tokens + n > token_budget:
                break
            need = -(-n // bs)
            if need > free:
                break
            batch.append((pending.popleft(), 0, take))
            tokens += take
            free -= need
        if not batch:
            if idle_sleep:
                time.sleep(idle_sleep)
            continue
        ids = tuple(f"pd-{requests[k][0]}" for k, _, _ in batch)
        chunks = tuple(requests[k][1][:, a:e] for k, a, e in batch)
        with torch.inference_mode():
            logits = paged_prefill_chunks(model, chunks, cache, ids)
            picked = ops.argmax_rows(logits) if logits.is_cuda else logits.argmax(dim=-1)
            first = picked.tolist()  # also waits for the KV writes
        finished = []
        for (k, a, e), tok in zip(batch, first):
            if e < requests[k][1].shape[1]:
                if a == 0:
                    started.append(k)
                done[k] = e
                continue
            if a > 0:
                started.remove(k)
                del done[k]
            finished.append((k, tok))
        if first_token_at is not None and finished:
            now = clock()
            for k, _ in finished:
                first_token_at[requests[k][0]] = now
        for k, tok in finished:
            index, prompt = requests[k]
            sid = f"pd-{index}"
            table = cache.get_block_table(sid)
            channels[route[k]].send([HANDOFF, index, prompt.shape[1], int(tok), len(table), 0, 0, 0, *table])
            sent[route[k]] += 1
            held[index] = sid
            stats.requests += 1
        stats.tokens += tokens
        stats.batches += 1
    for ch, n in zip(channels, sent):
        ch.send([DONE, n])
        ch.close()
    return stats


def run_decode(
    model,
    cache: PagedKVCache,
    channel: PairChannel,
    prompt_of: Callable[[int], torch.Tensor],
    config: GenerationConfig,
    max_batch_size: int,
    import_fn: Callable,
    vocab_size: int,
    *,
    idle_sleep: float = 0.0,
    clock: Callable[[], float] = time.perf_counter,
    timings: dict[int, tuple[float, float]] | None = None,
    graph_batches: int = 0,
) -> list[PagedRequest]:
    """Receive hand-offs, import their KV, and decode them with continuous batching.

    ``timings`` receives, per request index, the ``clock()`` times at which
    its hand-off arrived and at which it completed.  With ``graph_batches``
    the decode graphs of batch sizes 1 .. graph_batches are captured after
    the first decode step (the block table first sized for ``max_batch_size``
    sequences of the model's longest length), so that a batch size seen later
    does not stall its step with a capture.
    """
    sched = ContinuousBatchingScheduler(model, config, cache, max_batch_size)
    ready: deque[tuple[PagedRequest, torch.Tensor]] = deque()
    copies: deque[tuple[object, int]] = deque()
    requests: list[PagedRequest] = []
    received: dict[str, tuple[int, float]] = {}
    done = False
    bs = cache.block_size
    dtype = cache.keys.dtype
    while True:
        for msg in () if done else channel.poll(stop_after=DONE):
            if msg[0] == HANDOFF:
                index, length, token, nblk = msg[1], msg[2], msg[3], msg[4]
                sid = f"pd-{index}"
                if timings is not None:
                    received[sid] = (index, clock())
                event = import_fn(cache, sid, length, msg[HEADER_WORDS : HEADER_WORDS + nblk])
                prompt = prompt_of(index)
                required = (length + config.max_new_tokens - 1 + bs - 1) // bs
                request = PagedRequest(sequence_id=sid, prompt=prompt, required_blocks=required)
                logits = torch.zeros(vocab_size, dtype=dtype, device=cache.device)
                logits[token] = 1
                ready.append((request, logits))
                copies.append((event, index))
            elif msg[0] == DONE:
                done = True
        while copies and (copies[0][0] is None or copies[0][0].query()):
            channel.send([ACK, copies.popleft()[1]])
        while (
            ready
            and sched.active_count < max_batch_size
            and sched.reserved_blocks + ready[0][0].required_blocks <= sched.block_budget
        ):
            request, logits = ready.popleft()
            sched.add_prefilled_request(request, logits)
            requests.append(request)
        if sched.has_work:
            out = sched.step()
            if graph_batches and hasattr(model, "capture_decode_graphs"):
                cache.reserve_table(max_batch_size, -(-model.config.max_seq_len // bs))
                model.capture_decode_graphs(cache, range(1, graph_batches + 1))
                graph_batches = 0
            if timings is not None and out.terminal_requests:
                now = clock()
                for r in out.terminal_requests:
                    index, t0 = received[r.sequence_id]
                    timings[index] = (t0, now)
        elif done and not ready and not copies:
            break
        elif idle_sleep:
            time.sleep(idle_sleep)
    channel.close()
    return requests
