"""Seeded random-init Llama state dicts for the CPU oracle (test infrastructure only).

The random-init recipe used for every model-level parity case and for the
bench (applied the same way to the reference's module and to the engine's)
draws every tensor of the state dict in sorted-name order from one CPU
``torch.Generator``: norm weights are filled with 1, every other tensor with
N(0, std) in fp32, and a tied ``lm_head.weight`` shares ``embed.weight`` so
it is drawn once.  ``random_llama_state`` restates that recipe from the
architecture alone, so the bench's CPU legs and the tests can build the
oracle's weights without importing the product package.

State-dict names and shapes follow the reference module tree
(models/llama.py:95-125, layers/decoder.py:8-21, layers/attention.py:121-145,
layers/mlp.py:8-16, paths relative to the reference's src/nano_infer_engine/).
"""

from __future__ import annotations

import torch

# Llama-3.2-1B shape (reference models/llama.py:23-57 defaults)
LLAMA_1B = dict(
    vocab_size=128256,
    hidden_size=2048,
    mlp_inner_size=8192,
    num_layers=16,
    q_head_num=32,
    kv_head_num=8,
    norm_eps=1e-5,
    rope_type="llama3",
    rope_theta=500000.0,
    tie_word_embeddings=True,
)


def llama_state_shapes(config: dict) -> dict[str, tuple[int, ...]]:
    """Name -> shape of every state-dict entry (``lm_head.weight`` included, tied or not)."""
    h = config["hidden_size"]
    hd = h // config["q_head_num"]
    kv = config["kv_head_num"] * hd
    m = config["mlp_inner_size"]
    shapes: dict[str, tuple[int, ...]] = {"embed.weight": (config["vocab_size"], h)}
    for i in range(config["num_layers"]):
        p = f"decoders.{i}."
        shapes[p + "attn.q_proj.weight"] = (h, h)
        shapes[p + "attn.k_proj.weight"] = (kv, h)
        shapes[p + "attn.v_proj.weight"] = (kv, h)
        shapes[p + "attn.o_proj.weight"] = (h, h)
        shapes[p + "ffn.down_proj.weight"] = (h, m)
        shapes[p + "ffn.up_proj.weight"] = (m, h)
        shapes[p + "ffn.gate_proj.weight"] = (m, h)
        shapes[p + "pre_norm.weight"] = (h,)
        shapes[p + "post_norm.weight"] = (h,)
    shapes["final_rms.weight"] = (h,)
    shapes["lm_head.weight"] = (config["vocab_size"], h)
    return shapes


def random_llama_state(config: dict, seed: int, std: float = 0.02,
                       dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """Seeded N(0, std) state dict, norms = 1, drawn in sorted-name order (tied lm_head drawn once)."""
    tied = config.get("tie_word_embeddings", True)
    shapes = llama_state_shapes(config)
    gen = torch.Generator().manual_seed(seed)
    state: dict[str, torch.Tensor] = {}
    for name in sorted(shapes):
        if tied and name == "lm_head.weight":
            continue
        if name.endswith("norm.weight") or name.endswith("final_rms.weight"):
            state[name] = torch.ones(shapes[name], dtype=dtype)
        else:
            draw = torch.empty(shapes[name], dtype=torch.float32).normal_(0.0, std, generator=gen)
            state[name] = draw.to(dtype)
    if tied:
        state["lm_head.weight"] = state["embed.weight"]
    return state
