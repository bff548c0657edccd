"""Seeded input recipes shared by the golden generator and the tests.

Inputs are regenerated from these recipes (CPU torch RNG is deterministic
for a fixed torch version), so only the reference's OUTPUTS are stored as
fixtures.  Nothing here imports the reference or the product.
"""

from __future__ import annotations

import torch

# ------------------------------------------------------------ decode cases
DECODE_CASES = ("tiny_f32", "llama_bf16", "llama_f32")


def decode_case(name: str) -> dict:
    if name == "tiny_f32":
        # reference tests/test_paged_attention.py:59-98 shape (hd 3, bs 2, 4q/2kv)
        g = torch.Generator().manual_seed(1)
        q = torch.randn(3, 4, 3, generator=g)
        kc = torch.randn(2, 7, 2, 2, 3, generator=g)
        vc = torch.randn(2, 7, 2, 2, 3, generator=g)
        return dict(query=q, key_cache=kc, value_cache=vc,
                    tables=[[5, 1], [4, 0, 6], [2]], seq_lens=[3, 5, 2], layer=1)
    if name in ("llama_bf16", "llama_f32"):
        dtype = torch.bfloat16 if name == "llama_bf16" else torch.float32
        g = torch.Generator().manual_seed(3)
        pool, bs, hkv, hd, hq = 96, 16, 8, 64, 32
        seq_lens = [1, 15, 16, 17, 300, 33, 160]
        perm = torch.randperm(pool, generator=g).tolist()
        tables, at = [], 0
        for n in seq_lens:
            nb = (n + bs - 1) // bs
            tables.append(perm[at : at + nb])
            at += nb
        kc = torch.randn(2, pool, bs, hkv, hd, generator=g).to(dtype)
        vc = torch.randn(2, pool, bs, hkv, hd, generator=g).to(dtype)
        q = torch.randn(len(seq_lens), hq, hd, generator=g).to(dtype)
        return dict(query=q, key_cache=kc, value_cache=vc, tables=tables, seq_lens=seq_lens, layer=1)
    raise KeyError(name)


# ------------------------------------------------------ GQA ragged cases
RAGGED_CASES = ("gqa_bf16", "gqa_f32")


def ragged_case(name: str) -> dict:
    """One GroupedQueryAttention.forward_ragged call on a prefilled paged cache.

    Geometry: hidden 512, 8 q heads, 2 kv heads (head_dim 64), block 16.
    Requests: prefill chunks of 5/16/33 tokens at contexts 0/7/20 and two
    decode tokens at contexts 40/3 (prefill first, then decode, as the
    scheduler orders them).
    """
    dtype = torch.bfloat16 if name == "gqa_bf16" else torch.float32
    g = torch.Generator().manual_seed(11)
    hidden, hq, hkv, bs = 512, 8, 2, 16
    contexts = [0, 7, 20, 40, 3]
    qlens = [5, 16, 33, 1, 1]
    ids = ("req-a", "req-b", "req-c", "req-d", "req-e")
    weights = {
        n: (torch.randn(shape, generator=g) * 0.05).to(dtype)
        for n, shape in (
            ("q_proj.weight", (hidden, hidden)),
            ("k_proj.weight", (hkv * 64, hidden)),
            ("v_proj.weight", (hkv * 64, hidden)),
            ("o_proj.weight", (hidden, hidden)),
        )
    }
    # history K/V for the cached context of each request, [ctx, hkv, 64]
    history = [(torch.randn(c, hkv, 64, generator=g).to(dtype), torch.randn(c, hkv, 64, generator=g).to(dtype))
               for c in contexts]
    x = torch.randn(sum(qlens), hidden, generator=g).to(dtype)
    # allocation warm-up that makes the physical layout non-contiguous
    return dict(hidden=hidden, hq=hq, hkv=hkv, block_size=bs, num_blocks=48, contexts=contexts,
                qlens=qlens, ids=ids, weights=weights, history=history, x=x, dtype=dtype,
                rope_theta=500000.0, warmup=[("tmp-0", 20), ("tmp-1", 40)], release=["tmp-0"])


# ------------------------------------------------------- paging scenario
def paging_scenario() -> list[tuple]:
    """A scripted sequence of cache operations (ops are applied in order)."""
    return [
        ("ensure", "a", 5), ("ensure", "b", 17), ("ensure", "c", 1), ("release", "a"),
        ("ensure", "d", 33), ("ensure", "b", 40), ("advance", "b", 40), ("release", "c"),
        ("ensure", "e", 16), ("ensure", "a", 2), ("ensure", "d", 49), ("release", "b"),
        ("ensure", "f", 64), ("advance", "d", 49), ("ensure", "d", 50),
    ]


# ---------------------------------------------------------- model config
def config1_kwargs() -> dict:
    """BASELINE config 1 model (rope theta 5e5; plain RoPE; untied lm_head)."""
    return dict(vocab_size=1024, hidden_size=256, mlp_inner_size=1024, num_layers=2, q_head_num=4,
                kv_head_num=2, norm_eps=1e-5, rope_type="default", rope_theta=500000.0,
                tie_word_embeddings=False)


def config1_prompts() -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 1024, (1, n), generator=g) for n in (7, 33, 64, 100)]


CONFIG1_WEIGHT_SEED = 0
CONFIG1_STD = 0.02

# BASELINE config 2 (Llama-3.2-1B shape, bf16): the bench's seeded workload
CONFIG2_WEIGHT_SEED = 1234
CONFIG2_FULL_NEW_TOKENS = 256  # the full config-2 generation (dense reference golden)


def config2_prompts(num_requests: int = 16, seed: int = 1234) -> list[torch.Tensor]:
    """16 prompts, lengths U[128, 2048], ids U[0, 128256) (same draw as bench.py)."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(128, 2049, (num_requests,), generator=g).tolist()
    return [torch.randint(0, 128256, (1, n), generator=g) for n in lengths]


# ------------------------------------------------------------ P/D pipeline
# BASELINE config-1 model (fp32) behind the prefill/decode pipeline: six
# prompts, 16 new tokens, a decode pool small enough that the worst-case
# block reservation (not only the batch slots) holds requests back.
PD_PROMPT_LENS = (7, 33, 64, 100, 1, 45)
PD_NEW_TOKENS = 16
PD_MAX_BATCH = 3
PD_PREFILL_BLOCKS = 32
PD_DECODE_BLOCKS = 12
# pd_greedy_generate: two requests through shared caches, then one with EOS
PD_GREEDY_PROMPT_LENS = (33, 100)
PD_GREEDY_NEW_TOKENS = 12
PD_GREEDY_BLOCKS = 16
PD_GREEDY_EOS_INDEX = 4  # EOS = the token the first request generated at this index


def pd_prompts(lengths=PD_PROMPT_LENS, seed: int = 21) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 1024, (1, n), generator=g) for n in lengths]
