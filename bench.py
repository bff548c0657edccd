"""Benchmark of the B200 ragged-batch attention engine (one JSON line on rank 0).

Headline: output tokens/s of continuous batching at
Llama-3.2-1B shape on random-init bf16 weights (std 0.02): 16 requests,
prompts U[128, 2048], 256 greedy new tokens each, prefill chunk 128, at most
512 prefill tokens per step, block size 16, max model length 29600.  One
"step" = one full generation of that batch through the public scheduler API.

* ``value``   - tokens/s with prompts resident in HBM;
* ``e2e``     - the same through the public API from pinned HOST prompts,
                H2D of the prompts and D2H of every generated sequence inside
                the timed region;
* ``roofline``- the paged decode kernel on BASELINE config 3 (B=64, ctx
                U[512, 29600], 131072-block pool), algorithmic bytes / CUDA-
                event time vs the measured HBM copy bandwidth;
* ``cpu_baseline`` - the CPU oracle (restated reference forward) on a bounded
                sample of the same workload, extrapolated to tokens/s.

N GPUs (torchrun), N a multiple of k + 1: N/(k+1) P/D groups of one prefill
GPU feeding k decode GPUs behind the router (k = --pd-decode-per-prefill:
by default 3 when N is a multiple of 4, else 1; BASELINE config 5's
prompt-length distribution, the same 32 requests per decode GPU, closed
loop, weak scaling, max-over-ranks time); the prefill GPU hands requests off
and each decode GPU pulls their KV blocks over NVLink (CUDA IPC).  Other N:
independent replicas of the 1-GPU run.
``--impl reference`` times the reference algorithm on the host cores (the
oracle port; rank 0 only) for the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "output tok/s at Llama-3.2-1B shape"
UNIT = "tok/s"
SEED = 1234


# ------------------------------------------------------------------ helpers
def headline_config(args, world):
    """The N=1 / replica workload description, shared verbatim by both arms."""
    return {
        "workload": "config2: Llama-3.2-1B shape, 16 requests, prompts U[128,2048], 256 greedy new "
                    "tokens, prefill chunk 128, <=512 prefill tokens/step, block 16, max_model_len 29600",
        "global_batch": args.requests * world,
        "parallelism": f"replicas x{world}",
        "l2": "inputs larger than L2 (2.47 GB of weights streamed per decode step)",
    }


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--requests", type=int, default=16)
    p.add_argument("--new-tokens", type=int, default=256)
    p.add_argument("--decode-iters", type=int, default=20)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--only", choices=("all", "engine", "decode", "mixed", "pd-open", "linear"), default="all",
                   help="engine: headline run only; decode: config-3 decode micro-bench only; "
                        "mixed: config-4 mixed step only (profiling); pd-open: config 5 open loop "
                        "(Poisson arrivals, TTFT/TPOT, transfer GB/s; N >= 2, a multiple of k + 1)")
    p.add_argument("--pd-requests", type=int, default=512)
    p.add_argument("--pd-rate", type=float, default=20.0)
    p.add_argument("--pd-decode-per-prefill", type=int, default=None,
                   help="N >= 2: decode ranks fed by each prefill rank (1 = prefill/decode pairs); default 3 when "
                        "N is a multiple of 4 (one prefill GPU keeps three decode GPUs fed), else 1")
    p.add_argument("--decode-batch", type=int, default=64)
    p.add_argument("--decode-blocks", type=int, default=131072)
    return p.parse_args()


def llama_1b_config(max_seq_len=29600):
    from nano_infer_engine_b200.models.llama import LlamaConfig

    return LlamaConfig(max_seq_len=max_seq_len)


def workload(num_requests, seed=SEED):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(128, 2049, (num_requests,), generator=g).tolist()
    return [torch.randint(0, 128256, (1, n), generator=g) for n in lengths]


class ClockSampler:
    """NVML clocks / throttle reasons sampled every 100 ms while running."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
                get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
                    n, "nvmlDeviceGetCurrentClocksThrottleReasons")
                self.reasons |= get(self.handle) & ~0x1
            except Exception:
                pass
            time.sleep(0.1)

    def __enter__(self):
        if self.nvml:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.nvml:
            self.thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        busy = [s for s in self.samples if s > 500] or self.samples
        return {
            "sm_mhz": statistics.median(busy),
            "sm_max_mhz": self.max_mhz,
            "reasons": [name for bit, name in self.REASONS.items() if self.reasons & bit],
        }


# ---------------------------------------------------------- engine run
def build_engine(device):
    from nano_infer_engine_b200.models.llama import build_random_llama

    return build_random_llama(llama_1b_config(), SEED, 0.02, torch.bfloat16, device)


def make_cache(device, num_requests, max_tokens):
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    blocks = num_requests * (-(-max_tokens // 16)) + 64
    return PagedKVCache(blocks, 16, 16, 8, 64, torch.bfloat16, device)


def generate(model, cache, prompts, new_tokens):
    """One step: the whole batch through the public scheduler API."""
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler

    config = GenerationConfig(max_new_tokens=new_tokens, prefill_chunk_size=128, max_prefill_tokens_per_step=512)
    sched = ContinuousBatchingScheduler(model, config, cache, len(prompts))
    reqs = [sched.add_request(f"req-{i}", p) for i, p in enumerate(prompts)]
    sched.run_until_idle()
    return reqs


def time_engine(model, cache, prompts, new_tokens, steps, warmup, dist_ctx):
    from nano_infer_engine_b200 import ops

    for _ in range(warmup):
        generate(model, cache, prompts, new_tokens)
    torch.cuda.synchronize()
    barrier(dist_ctx)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.LAUNCHES
    start.record()
    for _ in range(steps):
        generate(model, cache, prompts, new_tokens)
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / 1e3, ops.LAUNCHES - launches0


def time_e2e(model, cache, host_prompts, new_tokens, steps, device):
    """Prompts start in pinned host memory; results are read back to the host."""
    h2d = sum(p.numel() * p.element_size() for p in host_prompts)
    d2h = 0
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        prompts = [p.to(device, non_blocking=True) for p in host_prompts]
        reqs = generate(model, cache, prompts, new_tokens)
        outs = [r.sequence.to("cpu") for r in reqs]
        d2h = sum(o.numel() * o.element_size() for o in outs)
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / 1e3, h2d, d2h


# ------------------------------------------------------ P/D pairs (N >= 2)
PD_REQUESTS_PER_GPU = 16


def pd_workload(num_requests, seed=SEED):
    """BASELINE config 5's prompt lengths: log-normal with mean 1024 (sigma 1), capped to [1, 8192]."""
    g = torch.Generator().manual_seed(seed + 5)
    lengths = torch.empty(num_requests, dtype=torch.float64).log_normal_(math.log(1024) - 0.5, 1.0, generator=g)
    lengths = lengths.round().clamp(1, 8192).long().tolist()
    return [torch.randint(0, 128256, (1, n), generator=g) for n in lengths]


class PDRank:
    """One rank of a P/D group: rank g*j prefills for the decode ranks
    g*j+1 .. g*j+k of its group (g = k + 1; k = 1 is a pair).

    The router (``assign_groups``, least outstanding prompt+output tokens)
    splits the job's requests over the groups and, inside a group, over its
    decode ranks, identically on every rank; the prefill rank's KV pool is
    mapped into each of its decode ranks with CUDA IPC and blocks are pulled
    with the block-copy kernel.
    """

    def __init__(self, dist_ctx, rank, world, device, model, host_prompts, new_tokens, decode_per_prefill=1):
        from nano_infer_engine_b200.generation.pd_disagg import (
            HEADER_WORDS,
            PipeChannel,
            assign_groups,
            gpu_import,
            open_peer_pool,
            publish_pool,
        )
        from nano_infer_engine_b200.paged_cache import PagedKVCache

        k = decode_per_prefill
        g = k + 1
        self.device = device
        self.model = model
        self.new_tokens = new_tokens
        self.prefill = rank % g == 0
        self.rank = rank
        head = rank - rank % g
        self.peers = [head + 1 + j for j in range(k)] if self.prefill else [head]
        self.store = dist_ctx.distributed_c10d._get_default_store()
        work = [p.shape[1] + new_tokens for p in host_prompts]
        slots = assign_groups(work, world // g, k)[rank // g]
        if self.prefill:
            self.route = {i: j for j, slot in enumerate(slots) for i in slot}
            self.mine = sorted(self.route)
        else:
            self.mine = slots[rank % g - 1]
        self.host = {i: host_prompts[i] for i in self.mine}
        self.resident = {i: p.to(device) for i, p in self.host.items()}
        longest = max(p.shape[1] for p in host_prompts)
        # the ranks of a group share a node: records go over pairs of named pipes
        self.channels = [PipeChannel(self.store, rank, peer, HEADER_WORDS + -(-longest // 16)) for peer in self.peers]
        blocks = sum(-(-(self.host[i].shape[1] + (0 if self.prefill else new_tokens)) // 16) for i in self.mine)
        self.cache = PagedKVCache(blocks + 64, 16, 16, 8, 64, torch.bfloat16, device)
        if self.prefill:
            publish_pool(self.store, rank, self.cache)
            self.remote = None
        else:
            self.remote = open_peer_pool(self.store, self.peers[0], self.cache)
            self.transfers = []
            self.pull = gpu_import(self.remote, self.transfers)
            # decode graphs for batch sizes up to graph_batches are captured during
            # the first (warm-up) pass, on a block table sized once for every run
            self.graph_batches = min(64, len(self.mine))
            self.cache.reserve_table(len(self.mine) + 8, -(-model.config.max_seq_len // 16))

    def step(self, e2e=False, indices=None, arrival=None, clock=time.perf_counter, record=None):
        """One pass over this pair's requests (``indices``: a subset, in order);
        returns (h2d bytes, d2h bytes, outputs).  ``arrival`` maps request index
        to seconds after the pass starts (open loop); ``record`` collects
        first-token times (prefill rank) or (hand-off, completion) times (decode rank)."""
        from nano_infer_engine_b200.generation.config import GenerationConfig
        from nano_infer_engine_b200.generation.pd_disagg import run_decode, run_prefill

        mine = self.mine if indices is None else indices
        if e2e:
            prompts = {i: self.host[i].to(self.device, non_blocking=True) for i in mine}
            h2d = sum(self.host[i].numel() * self.host[i].element_size() for i in mine)
        else:
            prompts, h2d = self.resident, 0
        if self.prefill:
            run_prefill(self.model, self.cache, self.channels, [(i, prompts[i]) for i in mine],
                        token_budget=4096, chunk_size=2048, route=[self.route[i] for i in mine], idle_sleep=0.0002,
                        clock=clock, arrival=None if arrival is None else [arrival[i] for i in mine],
                        first_token_at=record)
            return h2d, 0, None
        reqs = run_decode(self.model, self.cache, self.channels[0], prompts.__getitem__,
                          GenerationConfig(max_new_tokens=self.new_tokens), len(mine), self.pull,
                          self.model.config.vocab_size, idle_sleep=0.0002, clock=clock, timings=record,
                          graph_batches=self.graph_batches)
        if e2e:
            outs = [r.sequence.to("cpu") for r in reqs]
            return h2d, sum(o.numel() * o.element_size() for o in outs), outs
        return h2d, 0, reqs

    def close(self):
        from nano_infer_engine_b200.generation.pd_disagg import close_peer_pool, wait_pool_unmapped

        if self.remote is not None:
            close_peer_pool(self.store, self.rank, self.remote)
        else:
            for peer in self.peers:
                wait_pool_unmapped(self.store, peer)
        for channel in self.channels:
            channel.release()


def time_pd(pd, steps, warmup, dist_ctx, e2e=False):
    from nano_infer_engine_b200 import ops

    with torch.inference_mode():
        for _ in range(warmup):
            pd.step(e2e)
        torch.cuda.synchronize()
        barrier(dist_ctx)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches0 = ops.LAUNCHES
        h2d = d2h = 0
        start.record()
        for _ in range(steps):
            h2d, d2h, _ = pd.step(e2e)
        stop.record()
        torch.cuda.synchronize()
    elapsed = start.elapsed_time(stop) / 1e3
    totals = torch.tensor([ops.LAUNCHES - launches0, h2d, d2h], dtype=torch.float64, device=pd.device)
    dist_ctx.all_reduce(totals)
    return max_over_ranks(dist_ctx, elapsed, pd.device), [int(x) for x in totals.tolist()]


def pd_layout(args, world):
    """(k, groups): decode ranks per prefill rank and P/D groups at N = world, the
    rule both arms use (--pd-decode-per-prefill, else 3 when N is a multiple of 4,
    else 1); groups = 0 when N does not form groups (replicas)."""
    k = args.pd_decode_per_prefill if args.pd_decode_per_prefill is not None else (3 if world % 4 == 0 else 1)
    return k, (world // (k + 1) if world >= 2 and k >= 1 and world % (k + 1) == 0 else 0)


def pd_config(args, base, groups, k):
    """The N >= 2 P/D workload description, shared verbatim by both arms."""
    lens = [p.shape[1] for p in base]
    return {
        "workload": f"config5 P/D, closed loop: Llama-3.2-1B shape, the same {len(base)} requests per decode GPU "
                    f"(prompts log-normal mean 1024 capped 8192, per decode GPU sum {sum(lens)}, max {max(lens)}), "
                    f"{args.new_tokens} greedy new tokens; prefill batches <=4096 tokens in chunks <=2048; KV blocks "
                    "pulled over NVLink by the decode GPU",
        "global_batch": len(base) * groups * k,
        "parallelism": f"{groups} P/D groups of 1 prefill + {k} decode ranks behind the router",
        "l2": "inputs larger than L2 (2.47 GB of weights streamed per decode step)",
    }


def pd_job(decode_ranks, new_tokens):
    """The closed-loop job for ``decode_ranks`` decode GPUs: the same seeded
    32-request set (config 5's prompt-length distribution) for every decode
    rank, interleaved one copy per decode rank per request.  The
    least-outstanding-work router then hands every decode rank one copy of
    each request, so the per-decode-rank workload is identical at every N and
    P:D ratio (weak scaling on a fixed job per decode GPU)."""
    base = pd_workload(2 * PD_REQUESTS_PER_GPU)
    job = [p for p in base for _ in range(decode_ranks)]
    return base, job


def run_pd(args, dist_ctx, rank, local, device, world):
    """N >= 2: N/(k+1) groups of one prefill rank and k decode ranks behind the
    router (k = --pd-decode-per-prefill; 1 = pairs), weak scaling (the same
    32-request set per decode rank), closed loop: one step = every decode rank
    generates its batch."""
    k = args.pd_decode_per_prefill
    groups = world // (k + 1)
    model = build_engine(device)
    base, job = pd_job(groups * k, args.new_tokens)
    host = [p.pin_memory() for p in job]
    pd = PDRank(dist_ctx, rank, world, device, model, host, args.new_tokens, k)
    with ClockSampler(local) as clocks:
        elapsed, (launches, _, _) = time_pd(pd, args.steps, args.warmup, dist_ctx)
    value = len(host) * args.new_tokens * args.steps / elapsed
    e2e = None
    if not args.no_e2e:
        e2e_steps = max(2, args.steps)
        e2e_s, (_, h2d, d2h) = time_pd(pd, e2e_steps, 1, dist_ctx, e2e=True)
        e2e = {"value": len(host) * args.new_tokens * e2e_steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": h2d // e2e_steps, "d2h_bytes_per_step": d2h // e2e_steps}
    pd.close()
    del pd
    torch.cuda.empty_cache()
    roofline = None
    if rank == 0 and args.only == "all":
        dec = decode_config3(device, args.decode_iters, args.decode_batch, args.decode_blocks)
        peak, peak_kind = measured_peaks()
        achieved = dec["bytes"] / (dec["ms"] / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": ncu_traffic(), "kernel": "decode_tma_kernel + decode_combine_kernel",
                    "workload": f"config3 decode on rank 0: B=64, sum ctx {dec['sum_ctx']}, "
                                f"{dec['bytes']} algorithmic bytes/launch",
                    "ms_per_launch": dec["ms"], "peak_kind": f"{peak_kind} (hbm_gbs burst copy)"}
    barrier(dist_ctx)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC,
            "value": value,
            "per_group": value / groups,
            "per_decode_gpu": value / (groups * k),
            "per_gpu": value / world,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded prompts, random-init weights N(0, 0.02))",
            "config": pd_config(args, base, groups, k),
            "roofline": roofline,
            "cpu_baseline": None,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }))
    dist_ctx.barrier()
    dist_ctx.destroy_process_group()
    return 0


def pd_open_workload(num_requests, rate, seed=SEED):
    """Config 5: log-normal prompts and Poisson arrivals (seeded exponential gaps)."""
    prompts = pd_workload(num_requests, seed)
    g = torch.Generator().manual_seed(seed + 9)
    gaps = torch.empty(num_requests, dtype=torch.float64).exponential_(rate, generator=g)
    return prompts, gaps.cumsum(0).tolist()


def _pct(values, q):
    values = sorted(values)
    return values[min(len(values) - 1, int(q * len(values)))] if values else None


def run_pd_open(args, dist_ctx, rank, local, device, world):
    """Config 5 open loop on N/(k+1) P/D groups: output tok/s (arrival-capped), TTFT, TPOT, transfer GB/s."""
    k = args.pd_decode_per_prefill
    model = build_engine(device)
    host, arrival = pd_open_workload(args.pd_requests, args.pd_rate)
    host = [p.pin_memory() for p in host]
    pd = PDRank(dist_ctx, rank, world, device, model, host, args.new_tokens, k)
    with torch.inference_mode():
        pd.step(indices=pd.mine[:16])  # warm-up: graphs, workspaces, allocator
        if not pd.prefill:
            pd.transfers.clear()
        torch.cuda.synchronize()
        record = {}
        with ClockSampler(local) as clocks:
            # the sampler is up before the clock starts: arrivals, first tokens
            # and completions all use this rank's clock from t0
            barrier(dist_ctx)
            t0 = time.monotonic()
            pd.step(arrival=arrival, clock=lambda: time.monotonic() - t0, record=record)
            torch.cuda.synchronize()
            elapsed = time.monotonic() - t0
    elapsed = max_over_ranks(dist_ctx, elapsed, device)
    # gather per-request timings and transfer records on rank 0 through the store
    store = dist_ctx.distributed_c10d._get_default_store()
    if pd.prefill:
        mine = {i: record[i] - arrival[i] for i in pd.mine}
    else:
        moved = [(b, s.elapsed_time(e) / 1e3) for b, s, e in pd.transfers]
        tpot = {i: (t1 - t0_) / max(1, args.new_tokens - 1) for i, (t0_, t1) in record.items()}
        mine = {"tpot": tpot, "transfers": moved}
    store.set(f"pdopen/{rank}", json.dumps(mine))
    pd.close()
    barrier(dist_ctx)
    if rank == 0:
        ttft, tpot, moved = [], [], []
        for r in range(world):
            data = json.loads(store.get(f"pdopen/{r}"))
            if r % (k + 1) == 0:
                ttft.extend(data.values())
            else:
                tpot.extend(data["tpot"].values())
                moved.extend(data["transfers"])
        per = [b / t / 1e9 for b, t in moved if t > 0]
        print(json.dumps({
            "mode": "pd-open (config 5)",
            "n_gpus": world,
            "groups": world // (k + 1),
            "decode_per_prefill": k,
            "requests": args.pd_requests,
            "rate_req_s": args.pd_rate,
            "new_tokens": args.new_tokens,
            "output_tok_s": args.pd_requests * args.new_tokens / elapsed,
            "arrival_cap_tok_s": args.pd_rate * args.new_tokens,
            "duration_s": elapsed,
            "ttft_ms": {"p50": 1e3 * _pct(ttft, 0.5), "p90": 1e3 * _pct(ttft, 0.9), "p99": 1e3 * _pct(ttft, 0.99)},
            "tpot_ms": {"p50": 1e3 * _pct(tpot, 0.5), "p90": 1e3 * _pct(tpot, 0.9), "p99": 1e3 * _pct(tpot, 0.99)},
            "transfer": {"count": len(moved), "bytes_total": sum(b for b, _ in moved),
                         "gbs_median": _pct(per, 0.5), "gbs_aggregate": sum(b for b, _ in moved) /
                         max(1e-12, sum(t for _, t in moved)) / 1e9,
                         "note": "bytes of the copied blocks (K+V, all layers) / copy-kernel event time on the "
                                 "decode GPU; reads cross NVLink from the prefill GPU's pool"},
            "clocks": clocks.summary(),
        }))
    dist_ctx.barrier()
    dist_ctx.destroy_process_group()
    return 0


# ------------------------------------------------------ decode roofline
def config3_inputs(device, B=64, nb=131072):
    """BASELINE config 3 inputs (seeded): B requests, ctx U[512, 29600], block tables
    consecutive slices of a random permutation of an nb-block pool, 1 layer, N(0, 1)."""
    g = torch.Generator().manual_seed(0)
    bs = 16
    lens = torch.randint(512, 29601, (B,), generator=g).tolist()
    if sum(-(-n // bs) for n in lens) > nb:
        raise ValueError(f"decode pool of {nb} blocks cannot hold batch {B}")
    perm = torch.randperm(nb, generator=g)
    width = max(-(-n // bs) for n in lens)
    tables = torch.full((B, width), -1, dtype=torch.int32)
    at = 0
    for i, n in enumerate(lens):
        k = -(-n // bs)
        tables[i, :k] = perm[at : at + k].to(torch.int32)
        at += k
    gen = torch.Generator(device=device).manual_seed(0)
    kc = torch.randn((1, nb, bs, 8, 64), generator=gen, device=device, dtype=torch.bfloat16)
    vc = torch.randn((1, nb, bs, 8, 64), generator=gen, device=device, dtype=torch.bfloat16)
    q = torch.randn((B, 32, 64), generator=gen, device=device, dtype=torch.bfloat16)
    return {"q": q, "kc": kc, "vc": vc, "tables": tables, "lens": lens, "tables_d": tables.to(device),
            "lens_d": torch.tensor(lens, dtype=torch.int32, device=device)}


def decode_config3(device, iters, B=64, nb=131072):
    """B=64, ctx U[512, 29600], pool 131072 blocks, 1 layer."""
    from nano_infer_engine_b200 import ops

    bs = 16
    inp = config3_inputs(device, B, nb)
    q, kc, vc, tables_d, lens_d, lens = inp["q"], inp["kc"], inp["vc"], inp["tables_d"], inp["lens_d"], inp["lens"]
    out = torch.empty_like(q)
    for _ in range(3):
        ops.paged_decode(q, kc, vc, 0, tables_d, lens_d, out=out)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        ops.paged_decode(q, kc, vc, 0, tables_d, lens_d, out=out)
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / iters
    ops.check_device_errors(device)
    sum_ctx = sum(lens)
    algo_bytes = sum_ctx * 2048 + sum(-(-n // bs) for n in lens) * 4 + 2 * B * 32 * 64 * 2
    del kc, vc
    torch.cuda.empty_cache()
    return {"ms": ms, "bytes": algo_bytes, "sum_ctx": sum_ctx, "batch": B}


def config4_inputs(device):
    """BASELINE config 4 inputs (seeded): 8 prefill chunks of 128 at ctx U[0, 8192] then
    120 decode rows at ctx U[256, 16384], random block tables, 1 layer, N(0, 1); the
    ragged metadata comes from the packing kernel."""
    from nano_infer_engine_b200 import ops

    g = torch.Generator().manual_seed(4)
    bs = 16
    contexts = torch.randint(0, 8193, (8,), generator=g).tolist() + torch.randint(256, 16385, (120,), generator=g).tolist()
    qlens = [128] * 8 + [1] * 120
    lens = [c + q for c, q in zip(contexts, qlens)]
    nb = sum(-(-n // bs) for n in lens) + 64
    perm = torch.randperm(nb, generator=g)
    width = max(-(-n // bs) for n in lens)
    tables = torch.full((len(lens), width), -1, dtype=torch.int32)
    at = 0
    for i, n in enumerate(lens):
        k = -(-n // bs)
        tables[i, :k] = perm[at : at + k].to(torch.int32)
        at += k
    gen = torch.Generator(device=device).manual_seed(4)
    kc = torch.randn((1, nb, bs, 8, 64), generator=gen, device=device, dtype=torch.bfloat16)
    vc = torch.randn((1, nb, bs, 8, 64), generator=gen, device=device, dtype=torch.bfloat16)
    T = sum(qlens)
    q = torch.randn((T, 32, 64), generator=gen, device=device, dtype=torch.bfloat16)
    R = len(lens)
    plan = torch.tensor([list(range(R)), contexts, qlens], dtype=torch.int32).to(device)
    meta = ops.pack_ragged(plan, T, tables.to(device), bs, nb, num_decode=120, max_query_len=128)
    return {"q": q, "kc": kc, "vc": vc, "tables": tables, "contexts": contexts, "qlens": qlens, "lens": lens,
            "meta": meta}


def config4_prefill(inp, out):
    """The prefill rows of the config-4 step on the tcgen05 kernel (split-KV workspace)."""
    from nano_infer_engine_b200 import ops

    m = inp["meta"]
    ops.varlen_attention(inp["q"], inp["kc"], inp["vc"], 0, m.block_tables, m.seq_lens, m.query_start_loc, 128,
                         out=out, table_rows=m.table_rows, req_list=m.prefill_list, num_requests=8,
                         max_seq_len=max(inp["lens"][:8]))


def config4_decode(inp, out):
    """The decode rows of the config-4 step on the split-K decode kernel."""
    from nano_infer_engine_b200 import ops

    m = inp["meta"]
    ops.paged_decode(inp["q"], inp["kc"], inp["vc"], 0, m.block_tables, m.seq_lens, out=out,
                     table_rows=m.table_rows, q_rows=m.query_start_loc, req_list=m.decode_list, num_requests=120)


def mixed_config4(device, iters):
    """8 prefill chunks of 128 at ctx U[0, 8192] + 120 decode rows at
    ctx U[256, 16384] (prefill first), one layer of the Llama-1B attention shape.
    Times the tcgen05 varlen kernel (attention, cut segments merged in-kernel) and the
    decode kernels separately, each as `iters` calls replayed from a CUDA graph."""
    from nano_infer_engine_b200 import ops

    bs = 16
    inp = config4_inputs(device)
    contexts, lens = inp["contexts"], inp["lens"]
    out = torch.empty_like(inp["q"])

    def prefill():
        config4_prefill(inp, out)

    def decode():
        config4_decode(inp, out)

    res = {}
    for name, fn in (("prefill", prefill), ("decode", decode)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        # the calls are replayed from a CUDA graph so that the host-side work
        # of each eager call (argument checks, tensor-map encoding) is not timed
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(iters):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        res[name + "_ms"] = a.elapsed_time(b) / iters
        del graph
    ops.check_device_errors(device)
    flops = sum(4 * 64 * 32 * (128 * c + 128 * 129 // 2) for c in contexts[:8])
    kc, vc = inp["kc"], inp["vc"]
    dec_bytes = sum(lens[8:]) * 2048 + sum(-(-n // bs) for n in lens[8:]) * 4 + 2 * 120 * 32 * 64 * 2
    res.update(prefill_flops=flops, prefill_tflops=flops / (res["prefill_ms"] / 1e3) / 1e12,
               decode_bytes=dec_bytes, decode_gbs=dec_bytes / (res["decode_ms"] / 1e3) / 1e9,
               prefill_contexts=contexts[:8])
    del kc, vc, inp
    torch.cuda.empty_cache()
    return res


def linear_decode_shapes(device, m=16, copies=16, reps=4):
    """nie_linear against torch's cuBLAS GEMM on the decode projections of config 2.

    Each shape runs over `copies` distinct weight matrices (more bytes than
    L2 holds except for the smallest), replayed from a CUDA graph; the
    time per call is the graph time / calls.  Algorithmic bytes per call =
    the weight matrix (x and y are < 0.1 % of it).
    """
    from nano_infer_engine_b200 import ops

    peak, _ = measured_peaks()
    gen = torch.Generator(device=device).manual_seed(SEED)
    rows = []
    for name, n, k in (("qkv", 3072, 2048), ("o_proj", 2048, 2048), ("gate_up", 16384, 2048),
                       ("down_proj", 2048, 8192)):
        ws = [torch.randn(n, k, device=device, dtype=torch.bfloat16, generator=gen) * 0.02 for _ in range(copies)]
        x = torch.randn(m, k, device=device, dtype=torch.bfloat16, generator=gen)
        row = {"shape": name, "m": m, "n": n, "k": k, "weight_bytes": n * k * 2}
        for impl, fn in (("cublas", torch.nn.functional.linear), ("nie_linear", ops.linear_stream)):
            stream = torch.cuda.Stream(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                for w in ws:
                    fn(x, w)
                torch.cuda.synchronize(device)
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(reps):
                        for w in ws:
                            fn(x, w)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(device)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(5):
                graph.replay()
            t1.record()
            torch.cuda.synchronize(device)
            us = t0.elapsed_time(t1) * 1e3 / (5 * reps * copies)
            row[impl] = {"us": us, "GB/s": n * k * 2 / us / 1e3, "frac": n * k * 2 / us / 1e3 / peak}
            del graph
        ref = torch.nn.functional.linear(x, ws[0]).float()
        row["max_abs_diff_vs_cublas"] = (ops.linear_stream(x, ws[0]).float() - ref).abs().max().item()
        rows.append(row)
        del ws
        torch.cuda.empty_cache()
    ops.check_device_errors(device)
    return rows


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peaks():
    """(burst, sustained) dense bf16 TFLOP/s and their source."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["bf16_tflops"]), float(data.get("bf16_tflops_sustained", data["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


# Llama-3.2-1B: parameters streamed per decode step (embedding table read once, as the
# tied lm_head) and the per-token matmul parameters of the 16 decoder layers
LLAMA_1B_PARAMS = 128256 * 2048 + 16 * (2 * 2048 * 2048 + 2 * 512 * 2048 + 3 * 8192 * 2048)
LLAMA_1B_LAYER_PARAMS = 16 * (2 * 2048 * 2048 + 2 * 512 * 2048 + 3 * 8192 * 2048)
KV_BYTES_PER_TOKEN = 16 * 2 * 8 * 64 * 2  # all layers, K and V, bf16


def workload_roofline(prompt_lens, new_tokens, ms_per_generation):
    """Ideal time of one config-2 generation on this GPU and the measured fraction of it.

    Decode (HBM-bound): the first token of each request comes from its prefill;
    each of the other new_tokens - 1 forwards streams every weight once per step
    (batched over the requests) and reads the request's cached KV (context
    prompt + s at step s).  Prefill (tensor-bound): 2 x layer parameters per
    prompt token, plus causal attention 4 x 64 x 32 x L(L+1)/2 per layer, plus
    one lm_head row per request.  Ideal = bytes / HBM peak + FLOPs / sustained
    bf16 peak (the step runs for seconds under the power cap).
    """
    hbm, _ = measured_peaks()
    _, sustained, kind = measured_tensor_peaks()
    steps = new_tokens - 1
    decode_bytes = steps * LLAMA_1B_PARAMS * 2 + sum(
        sum(L + s for s in range(1, new_tokens)) for L in prompt_lens) * KV_BYTES_PER_TOKEN
    prefill_flops = sum(2 * LLAMA_1B_LAYER_PARAMS * L + 16 * 4 * 64 * 32 * L * (L + 1) // 2
                        + 2 * 128256 * 2048 for L in prompt_lens)
    ideal_s = decode_bytes / (hbm * 1e9) + prefill_flops / (sustained * 1e12)
    return {
        "bound": "hbm (decode steps) + tensor (prefill)",
        "ideal_ms": ideal_s * 1e3,
        "measured_ms": ms_per_generation,
        "frac": ideal_s * 1e3 / ms_per_generation,
        "decode_bytes": decode_bytes,
        "prefill_flops": prefill_flops,
        "peaks": {"hbm_gbs": hbm, "bf16_tflops_sustained": sustained, "kind": kind},
        "note": "ideal = algorithmic decode bytes / HBM peak + prefill FLOPs / sustained bf16 peak, "
                "per generation of the batch; frac = ideal / measured",
    }


def ncu_traffic():
    path = ROOT / "profiles" / "decode_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


# ------------------------------------------------------------ CPU baseline
def cpu_sample(prompts, model_cpu_state, threads):
    """Reference algorithm (oracle port) on the host: one 512-token prefill step and
    one 16-token decode step at the workload's context lengths; extrapolated to the
    whole run (ceil(sum(prompt)/512) prefill steps + (new_tokens) decode steps)."""
    from oracle.engine import OracleCache, OracleLlama
    from oracle.weights import LLAMA_1B

    torch.set_num_threads(threads)
    cfg = LLAMA_1B
    model = OracleLlama(model_cpu_state, cfg)
    lens = [p.shape[1] for p in prompts]
    blocks = sum(-(-(n + 1) // 16) for n in lens) + 64
    hd = cfg["hidden_size"] // cfg["q_head_num"]
    cache = OracleCache(blocks, 16, cfg["num_layers"], cfg["kv_head_num"], hd, torch.bfloat16)
    ids = [f"r{i}" for i in range(len(prompts))]
    # contexts as if each prompt were already cached (values do not affect time)
    for s, n in zip(ids, lens):
        cache.tables.ensure_capacity(s, n)
        cache.tables.advance(s, n)
    with torch.inference_mode():
        # one prefill step: 4 chunks of 128 tokens at the first 4 requests' contexts
        t0 = time.perf_counter()
        pf_ids = ids[:4]
        model.forward_ragged(torch.randint(0, 128256, (512,)), pf_ids, [128] * 4, cache, last_only=True)
        t_pf = time.perf_counter() - t0
        t0 = time.perf_counter()
        model.forward_ragged(torch.randint(0, 128256, (len(ids),)), ids, [1] * len(ids), cache, last_only=True)
        t_dec = time.perf_counter() - t0
    return t_pf, t_dec


def cpu_sample_pd(prompts, model_cpu_state, threads):
    """The P/D job's reference algorithm (oracle port) on the host: the first
    prefill batch of a decode GPU's requests (<= 4096 tokens, prompts in
    chunks of <= 2048, as the prefill rank forms it) and one decode step of
    all its requests at their prompt contexts.  Returns (seconds, tokens) of
    the batch and the decode step's seconds."""
    from oracle.engine import OracleCache, OracleLlama
    from oracle.weights import LLAMA_1B

    torch.set_num_threads(threads)
    cfg = LLAMA_1B
    model = OracleLlama(model_cpu_state, cfg)
    lens = [p.shape[1] for p in prompts]
    blocks = 2 * sum(-(-(n + 1) // 16) for n in lens) + 64
    hd = cfg["hidden_size"] // cfg["q_head_num"]
    cache = OracleCache(blocks, 16, cfg["num_layers"], cfg["kv_head_num"], hd, torch.bfloat16)
    batch, chunks, tokens = [], [], 0
    for i, n in enumerate(lens):
        take = min(n, 2048, 4096 - tokens)
        if take <= 0:
            break
        batch.append(f"p{i}")
        chunks.append(take)
        tokens += take
    ids = [f"r{i}" for i in range(len(prompts))]
    for s_, n in zip(ids, lens):  # decode contexts: every prompt cached (values do not affect time)
        cache.tables.ensure_capacity(s_, n)
        cache.tables.advance(s_, n)
    with torch.inference_mode():
        t0 = time.perf_counter()
        model.forward_ragged(torch.randint(0, 128256, (tokens,)), batch, chunks, cache, last_only=True)
        t_pf = time.perf_counter() - t0
        t0 = time.perf_counter()
        model.forward_ragged(torch.randint(0, 128256, (len(ids),)), ids, [1] * len(ids), cache, last_only=True)
        t_dec = time.perf_counter() - t0
    return t_pf, tokens, t_dec


def cpu_baseline(prompts, new_tokens, state):
    threads = os.cpu_count() or 1
    t_pf, t_dec = cpu_sample(prompts, state, threads)
    n_pf = math.ceil(sum(p.shape[1] for p in prompts) / 512)
    total = n_pf * t_pf + new_tokens * t_dec
    tokens = len(prompts) * new_tokens
    return {
        "value": tokens / total,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": (f"oracle forward on host: one 512-token prefill step ({t_pf:.2f}s) and one "
                   f"{len(prompts)}-token decode step ({t_dec:.2f}s) at the workload's contexts; "
                   f"extrapolated to {n_pf} prefill + {new_tokens} decode steps"),
    }


def cpu_state_for_oracle():
    """The engine's random-init weights, rebuilt by the oracle (no product import: the
    reference arm must not load this package or its native library)."""
    from oracle.weights import LLAMA_1B, random_llama_state

    return random_llama_state(LLAMA_1B, SEED, 0.02, torch.bfloat16)


# --------------------------------------------------------------- dist
def init_dist(n):
    if n <= 1 or "RANK" not in os.environ:
        return None
    import datetime

    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist


def barrier(dist_ctx):
    if dist_ctx is not None:
        dist_ctx.barrier()


def max_over_ranks(dist_ctx, value, device):
    if dist_ctx is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist_ctx.all_reduce(t, op=dist_ctx.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------ reference
def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return 0
    state = cpu_state_for_oracle()
    threads = os.cpu_count() or 1
    k, groups = pd_layout(args, args.gpus)
    if groups:
        # the product arm's N >= 2 workload: the P/D closed loop, one host doing
        # every decode GPU's share in turn (the rate does not depend on N)
        prompts = pd_workload(2 * PD_REQUESTS_PER_GPU)
        config = pd_config(args, prompts, groups, k)

        def one_step():
            t_pf, pf_tokens, t_dec = cpu_sample_pd(prompts, state, threads)
            prefill_s = t_pf * sum(p.shape[1] for p in prompts) / pf_tokens
            return len(prompts) * args.new_tokens / (prefill_s + args.new_tokens * t_dec)

        sample = ("oracle port of the reference forward (torch on the host cores, no product code loaded); "
                  "each step times one P/D prefill batch (<=4096 tokens, chunks <=2048) and one decode step of "
                  f"the {len(prompts)} requests of a decode GPU at their prompt contexts and extrapolates to that "
                  f"GPU's job (its prompt tokens + {args.new_tokens} decode steps); median over steps")
    else:
        prompts = workload(args.requests)
        config = headline_config(args, max(1, args.gpus))

        def one_step():
            t_pf, t_dec = cpu_sample(prompts, state, threads)
            n_pf = math.ceil(sum(p.shape[1] for p in prompts) / 512)
            return len(prompts) * args.new_tokens / (n_pf * t_pf + args.new_tokens * t_dec)

        sample = ("oracle port of the reference forward (torch on the host cores, no product code loaded); "
                  "each step times one 512-token prefill step (4 chunks of 128) and one 16-request decode step "
                  "at the workload's prompt contexts and extrapolates to the whole generation "
                  f"(ceil(sum(prompt)/512) prefill + {args.new_tokens} decode steps); median over steps")
    for _ in range(args.warmup):
        one_step()
    values = []
    t_start = time.perf_counter()
    for _ in range(args.steps):
        values.append(one_step())
    wall = time.perf_counter() - t_start
    value = statistics.median(values)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": wall / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded prompts, random-init weights N(0, 0.02))",
        "config": config,
        "sample": sample,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------ main
def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    dist_ctx = init_dist(args.gpus)
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    import __graft_entry__

    if rank == 0 or dist_ctx is None:
        __graft_entry__.build()
    barrier(dist_ctx)
    world = dist_ctx.get_world_size() if dist_ctx else 1
    if args.pd_decode_per_prefill is None:
        args.pd_decode_per_prefill = 3 if world % 4 == 0 else 1
    group = args.pd_decode_per_prefill + 1
    if args.pd_decode_per_prefill < 1:
        raise SystemExit("--pd-decode-per-prefill must be >= 1")
    if world >= 2 and world % group == 0 and args.only == "pd-open":
        return run_pd_open(args, dist_ctx, rank, local, device, world)
    if args.only == "pd-open":
        raise SystemExit("--only pd-open needs a multiple of (--pd-decode-per-prefill + 1) GPUs >= 2 under torchrun")
    if world >= 2 and world % group == 0 and args.only in ("all", "engine"):
        return run_pd(args, dist_ctx, rank, local, device, world)
    if args.only == "decode":
        dec = decode_config3(device, args.decode_iters, args.decode_batch, args.decode_blocks)
        peak, _ = measured_peaks()
        gbs = dec["bytes"] / (dec["ms"] / 1e3) / 1e9
        print(json.dumps({"decode_ms": dec["ms"], "algorithmic_bytes": dec["bytes"], "GB/s": gbs,
                          "frac": gbs / peak, "batch": dec["batch"], "sum_ctx": dec["sum_ctx"]}))
        return 0
    if args.only == "mixed":
        print(json.dumps(mixed_config4(device, args.decode_iters)))
        return 0
    if args.only == "linear":
        for row in linear_decode_shapes(device):
            print(json.dumps(row))
        return 0
    model = build_engine(device)
    host_prompts = [p.pin_memory() for p in workload(args.requests)]
    prompts = [p.to(device) for p in host_prompts]
    cache = make_cache(device, args.requests, 2048 + args.new_tokens)

    with ClockSampler(local) as clocks:
        elapsed, launches = time_engine(model, cache, prompts, args.new_tokens, args.steps, args.warmup, dist_ctx)
    elapsed = max_over_ranks(dist_ctx, elapsed, device)
    world = dist_ctx.get_world_size() if dist_ctx else 1
    tokens = args.requests * args.new_tokens * args.steps * world
    value = tokens / elapsed

    e2e = None
    if not args.no_e2e:
        e2e_s, h2d, d2h = time_e2e(model, cache, host_prompts, args.new_tokens, max(2, args.steps), device)
        e2e_s = max_over_ranks(dist_ctx, e2e_s, device)
        e2e = {"value": args.requests * args.new_tokens * max(2, args.steps) * world / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    del cache
    torch.cuda.empty_cache()
    if args.only == "engine":
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "e2e": e2e, "gpu_launches": launches,
                              "ms_per_step": elapsed / args.steps * 1e3, "clocks": clocks.summary()}))
        return 0
    dec = decode_config3(device, args.decode_iters, args.decode_batch, args.decode_blocks)
    peak, peak_kind = measured_peaks()
    achieved = dec["bytes"] / (dec["ms"] / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": ncu_traffic(), "kernel": "decode_tma_kernel + decode_combine_kernel",
                "workload": f"config3 decode: B=64, sum ctx {dec['sum_ctx']}, {dec['bytes']} algorithmic bytes/launch",
                "ms_per_launch": dec["ms"], "peak_kind": f"{peak_kind} (hbm_gbs burst copy)"}

    mixed = mixed_config4(device, args.decode_iters)
    burst, _, tkind = measured_tensor_peaks()
    roofline_prefill = {"bound": "tensor", "achieved": mixed["prefill_tflops"], "peak": burst, "unit": "TFLOP/s",
                        "frac": mixed["prefill_tflops"] / burst, "kernel": "prefill_tc_kernel (cut segments merged in-kernel)",
                        "workload": f"config4 prefill rows: 8 x 128 queries at contexts {mixed['prefill_contexts']}, "
                                    f"{mixed['prefill_flops']} causal FLOPs/call",
                        "ms_per_launch": mixed["prefill_ms"], "peak_kind": f"{tkind} (bf16_tflops burst)",
                        "decode_rows_gbs": mixed["decode_gbs"]}
    roofline_workload = workload_roofline([p.shape[1] for p in host_prompts], args.new_tokens,
                                          elapsed / args.steps * 1e3)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        del model
        torch.cuda.empty_cache()
        cpu = cpu_baseline(workload(args.requests), args.new_tokens, cpu_state_for_oracle())

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded prompts, random-init weights N(0, 0.02))",
            "config": headline_config(args, world),
            "roofline": roofline,
            "roofline_workload": roofline_workload,
            "roofline_prefill": roofline_prefill,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line))
    if dist_ctx is not None:
        dist_ctx.barrier()
        dist_ctx.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
