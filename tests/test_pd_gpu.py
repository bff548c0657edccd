"""P/D disaggregation across processes (and across GPUs where the box has two).

* ``transfer_sequence`` inside one process, cuda:0 -> cuda:1 (the block-copy
  kernel writing into the peer's pool over NVLink); skipped on one GPU;
* a prefill process and a decode process (on cuda:0 and cuda:1, or both on
  cuda:0 when the box has one GPU): the decode process maps the prefill
  process's pool with CUDA IPC and pulls each request's blocks with the same
  kernel.  No kernel of one process waits on the other (the channel is on the
  host), so sharing one GPU is safe.  The KV bytes on both sides must be
  identical, and the greedy tokens must equal the reference's own P/D
  scheduler run on the same model and prompts (tests/golden/pd_tokens.json,
  config-1 model in fp32).  Two passes over the same requests reuse the
  channel, both pools and the sequence ids.
"""

import json
import socket
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import recipes

pytestmark = pytest.mark.gpu

NEW_TOKENS = recipes.PD_NEW_TOKENS
PASSES = 2
PREFILL_BLOCKS = 12  # holds a few prompts at a time: later batches wait for ACKs
GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "pd_tokens.json").read_text())


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def _devices():
    """(prefill device, decode device): two GPUs when present, else both on cuda:0."""
    return (0, 1) if torch.cuda.device_count() >= 2 else (0, 0)


def _model(device):
    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    cfg = LlamaConfig(**recipes.config1_kwargs())
    return build_random_llama(cfg, recipes.CONFIG1_WEIGHT_SEED, recipes.CONFIG1_STD, torch.float32, device), cfg


def _prompts(cfg):
    return recipes.pd_prompts()


def test_transfer_sequence_between_devices_is_bit_exact():
    _need_two_gpus()
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.paged_cache import PagedKVCache, transfer_sequence

    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    src = PagedKVCache(64, 16, 3, 2, 64, torch.bfloat16, d0)
    dst = PagedKVCache(64, 16, 3, 2, 64, torch.bfloat16, d1)
    dst.ensure_capacity("other", 70)  # destination block ids differ from the source's
    dst.keys.normal_()  # stale data in the blocks the transfer will reuse
    dst.values.normal_()
    dst.release("other")
    n = 45
    src.ensure_capacity("s", n)
    g = torch.Generator(device=d0).manual_seed(0)
    for layer in range(3):
        k = torch.randn(n, 2, 64, generator=g, device=d0).to(torch.bfloat16)
        v = torch.randn(n, 2, 64, generator=g, device=d0).to(torch.bfloat16)
        src.write(layer, "s", 0, k, v)
    src.advance("s", n)
    transfer_sequence(src, dst, "s")
    ops.check_device_errors(d0)
    ops.check_device_errors(d1)
    assert dst.get_sequence_length("s") == n
    for layer in range(3):
        ks, vs = src.gather(layer, "s", n)
        kd, vd = dst.gather(layer, "s", n)
        assert torch.equal(ks.cpu(), kd.cpu()) and torch.equal(vs.cpu(), vd.cpu())
    last = dst.get_block_table("s")[-1]
    assert not dst.keys[:, last, n % 16 :].any() and not dst.values[:, last, n % 16 :].any()


def _pair_worker(rank, port, out, devices):
    from nano_infer_engine_b200 import ops
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.pd_disagg import (
        HEADER_WORDS,
        PairChannel,
        close_peer_pool,
        gpu_import,
        open_peer_pool,
        publish_pool,
        run_decode,
        run_prefill,
        wait_pool_unmapped,
    )
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    torch.cuda.set_device(devices[rank])
    dev = torch.device("cuda", devices[rank])
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=120))
    model, cfg = _model(dev)
    prompts = [p.to(dev) for p in _prompts(cfg)]
    channel = PairChannel(store, rank, 1 - rank, HEADER_WORDS + 64)
    layers = cfg.num_layers
    saved = {}

    def record(cache, sid, n):
        saved[sid] = [tuple(t.cpu() for t in cache.gather(li, sid, n)) for li in range(layers)]

    if rank == 0:
        cache = PagedKVCache(PREFILL_BLOCKS, 16, layers, cfg.kv_head_num, cfg.head_dim, torch.float32, dev)
        publish_pool(store, 0, cache)
        release = cache.release

        def release_and_record(sid):
            record(cache, sid, cache.get_sequence_length(sid))
            release(sid)

        cache.release = release_and_record
        with torch.inference_mode():
            for _ in range(PASSES):  # passes reuse the channel, both pools and the sequence ids
                stats = run_prefill(model, cache, channel, list(enumerate(prompts)), token_budget=96,
                                    idle_sleep=0.0005)
        ops.check_device_errors(dev)
        wait_pool_unmapped(store, 1)
        result = {"kv": saved, "batches": stats.batches, "free": cache.allocator.free_block_count}
    else:
        cache = PagedKVCache(256, 16, layers, cfg.kv_head_num, cfg.head_dim, torch.float32, dev)
        remote = open_peer_pool(store, 0, cache)
        pull = gpu_import(remote)

        def pull_and_record(c, sid, length, src_blocks):
            event = pull(c, sid, length, src_blocks)
            event.synchronize()
            record(c, sid, length)
            return event

        with torch.inference_mode():
            for _ in range(PASSES):
                reqs = run_decode(model, cache, channel, lambda i: prompts[i],
                                  GenerationConfig(max_new_tokens=NEW_TOKENS), 4, pull_and_record, cfg.vocab_size,
                                  idle_sleep=0.0005)
        ops.check_device_errors(dev)
        close_peer_pool(store, 1, remote)
        result = {
            "kv": saved,
            "tokens": {r.sequence_id: r.sequence[0].tolist() for r in reqs},
            "free": cache.allocator.free_block_count,
        }
    torch.save(result, f"{out}.{rank}")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_prefill_decode_pair_processes_match_reference_golden(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    devices = _devices()
    path = str(tmp_path / "pair")
    mp.start_processes(_pair_worker, args=(_free_port(), path, devices), nprocs=2, start_method="spawn", join=True)
    pre = torch.load(path + ".0")
    dec = torch.load(path + ".1")
    assert pre["batches"] > 1
    assert pre["free"] == PREFILL_BLOCKS and dec["free"] == 256
    ids = [f"pd-{i}" for i in range(len(recipes.PD_PROMPT_LENS))]
    assert sorted(pre["kv"]) == sorted(dec["kv"]) == sorted(ids)
    for sid, layers in pre["kv"].items():
        for (kp, vp), (kd, vd) in zip(layers, dec["kv"][sid]):
            assert torch.equal(kp, kd) and torch.equal(vp, vd), sid
    prompts = recipes.pd_prompts()
    want = {sid: p[0].tolist() + GOLDEN["scheduler"]["tokens"][sid] for sid, p in zip(ids, prompts)}
    assert dec["tokens"] == want
