"""P/D disaggregation on two GPUs.

* ``transfer_sequence`` inside one process, cuda:0 -> cuda:1 (the block-copy
  kernel writing into the peer's pool over NVLink);
* a prefill process on cuda:0 and a decode process on cuda:1: the decode
  process maps the prefill pool with CUDA IPC and pulls each request's blocks
  with the same kernel.  The KV bytes on both sides must be identical and
  the greedy tokens must equal a single-GPU run of the same model (fp32, so
  that batching differences cannot flip a token).  Two passes over the same
  requests reuse the channel, both pools and the sequence ids.

Both tests skip on a box with fewer than two GPUs.
"""

import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

PROMPT_LENS = (5, 40, 77, 16, 130, 300, 1, 64)
NEW_TOKENS = 12
PASSES = 2


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def _model(device):
    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama

    cfg = LlamaConfig(vocab_size=512, hidden_size=512, mlp_inner_size=1024, num_layers=2, q_head_num=8,
                      kv_head_num=2, max_seq_len=4096)
    return build_random_llama(cfg, 11, 0.02, torch.float32, device), cfg


def _prompts(cfg):
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, cfg.vocab_size, (1, n), generator=g) for n in PROMPT_LENS]


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


def _pair_worker(rank, port, out):
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

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=120))
    model, cfg = _model(dev)
    prompts = [p.to(dev) for p in _prompts(cfg)]
    channel = PairChannel(store, rank, 1 - rank, HEADER_WORDS + 64)
    layers = cfg.num_layers
    saved = {}

    def record(cache, sid, n):
        saved[sid] = [tuple(t.cpu() for t in cache.gather(li, sid, n)) for li in range(layers)]

    if rank == 0:
        # 40 blocks hold a few prompts at a time: later batches wait for ACKs
        cache = PagedKVCache(40, 16, layers, cfg.kv_head_num, cfg.head_dim, torch.float32, dev)
        publish_pool(store, 0, cache)
        release = cache.release

        def release_and_record(sid):
            record(cache, sid, cache.get_sequence_length(sid))
            release(sid)

        cache.release = release_and_record
        with torch.inference_mode():
            for _ in range(PASSES):  # passes reuse the channel, both pools and the sequence ids
                stats = run_prefill(model, cache, channel, list(enumerate(prompts)), token_budget=256,
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


def test_prefill_decode_pair_processes_match_single_gpu(tmp_path):
    _need_two_gpus()
    from nano_infer_engine_b200.generation.config import GenerationConfig
    from nano_infer_engine_b200.generation.scheduler import ContinuousBatchingScheduler
    from nano_infer_engine_b200.paged_cache import PagedKVCache

    path = str(tmp_path / "pair")
    mp.start_processes(_pair_worker, args=(_free_port(), path), nprocs=2, start_method="spawn", join=True)
    pre = torch.load(path + ".0")
    dec = torch.load(path + ".1")
    assert pre["batches"] > 1
    assert pre["free"] == 40 and dec["free"] == 256
    assert sorted(pre["kv"]) == sorted(dec["kv"]) == sorted(f"pd-{i}" for i in range(len(PROMPT_LENS)))
    for sid, layers in pre["kv"].items():
        for (kp, vp), (kd, vd) in zip(layers, dec["kv"][sid]):
            assert torch.equal(kp, kd) and torch.equal(vp, vd), sid

    dev = torch.device("cuda", 0)
    model, cfg = _model(dev)
    cache = PagedKVCache(256, 16, cfg.num_layers, cfg.kv_head_num, cfg.head_dim, torch.float32, dev)
    sched = ContinuousBatchingScheduler(model, GenerationConfig(max_new_tokens=NEW_TOKENS), cache, 4)
    reqs = [sched.add_request(f"pd-{i}", p.to(dev)) for i, p in enumerate(_prompts(cfg))]
    with torch.inference_mode():
        sched.run_until_idle()
    want = {r.sequence_id: r.sequence[0].tolist() for r in reqs}
    assert dec["tokens"] == want
