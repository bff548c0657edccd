"""Llama-3.2 model with the reference's API, running attention on the sm_100a path.

Reference: nano_infer_engine/models/llama.py.  ``LlamaConfig`` and the
state-dict names are identical, so a checkpoint or random state dict loads
into either engine.  All paged entry points (``forward`` with a
``PagedKVCache`` and ``forward_ragged``) are executed as one *ragged step*:

1. host: validation and block allocation (``ensure_capacity``) exactly as
   the reference, in the same order, so block tables are bit-identical;
2. device: kernel (a) expands the per-request plan into positions, slot
   mapping, query_start_loc and decode/prefill lists;
3. per layer: projections + RoPE (torch), slot write (b), decode (c) and
   varlen (d) attention, o_proj and MLP (torch);
4. host: ``advance`` per sequence.

Logits are computed for every token, as the reference returns them, unless
the caller (this package's ``paged_prefill``/``paged_prefill_chunks``) marks
that only each request's last row is read; then only those rows go through
the final norm and ``lm_head`` (reference llama.py:391 computes all rows
and paged_prefill.py:154-155 keeps the last ones).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

from .. import ops
from ..layers.attention import fused_weight
from ..layers.decoder import Llama3Decoder
from ..layers.rms_norm import RmsNorm
from ..layers.rope import Rope, RopeScale
from ..paged_cache import PagedKVCache

# Attribute a caller sets on the input-id (or query_start_loc) tensor to ask
# for last-row logits only; the returned logits carry LAST_ROWS_DONE = True
# when the request was honoured.
LAST_ROWS_ONLY = "_nie_last_rows_only"
LAST_ROWS_DONE = "_nie_last_rows"
HOST_BOUNDARIES = "_nie_host_boundaries"


@dataclass
class RopeScalingConfig:
    factor: float = 32.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass
class LlamaConfig:
    """Same fields and defaults as reference models/llama.py:23-70."""

    vocab_size: int = 128256
    hidden_size: int = 2048
    mlp_inner_size: int = 8192
    num_layers: int = 16
    q_head_num: int = 32
    kv_head_num: int = 8
    norm_eps: float = 1e-5
    rope_type: str = "llama3"
    rope_theta: float = 500000.0
    max_seq_len: int = 131072
    rope_scaling: RopeScalingConfig = field(default_factory=RopeScalingConfig)
    hidden_act: str = "silu"
    attention_bias: bool = False
    mlp_bias: bool = False
    attention_dropout: float = 0.0
    tie_word_embeddings: bool = True
    initializer_range: float = 0.02
    bos_token_id: int = 128000
    eos_token_id: int = 128001

    def __post_init__(self) -> None:
        assert self.hidden_size % self.q_head_num == 0
        assert self.q_head_num % self.kv_head_num == 0
        assert self.head_dim % 2 == 0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.q_head_num

    @property
    def group_num(self) -> int:
        return self.q_head_num // self.kv_head_num


def build_rope(config: LlamaConfig) -> Rope:
    if config.rope_type == "default":
        return Rope(dim=config.head_dim, theta_base=config.rope_theta)
    if config.rope_type == "llama3":
        s = config.rope_scaling
        return RopeScale(
            dim=config.head_dim,
            theta_base=config.rope_theta,
            scaling_factor=s.factor,
            low_freq_factor=s.low_freq_factor,
            high_freq_factor=s.high_freq_factor,
            original_max_position_embeddings=s.original_max_position_embeddings,
        )
    raise ValueError(f"Unsupported rope type: {config.rope_type}")


def init_random_weights_(model: nn.Module, seed: int, std: float = 0.02) -> nn.Module:
    """Seeded N(0, std) weights, norms = 1, identical for any module with the same state-dict names.

    Tensors are visited in sorted name order and drawn in fp32 on the CPU from
    one ``torch.Generator``; tied tensors are filled once.  Works on this
    package's model and on the reference's (same names), which is how both
    engines get identical random-init weights.
    """
    gen = torch.Generator().manual_seed(seed)
    state = model.state_dict()
    seen: set[int] = set()
    with torch.no_grad():
        for name in sorted(state):
            tensor = state[name]
            if tensor.data_ptr() in seen:
                continue
            seen.add(tensor.data_ptr())
            if name.endswith("norm.weight") or name.endswith("final_rms.weight"):
                tensor.fill_(1.0)
            else:
                draw = torch.empty(tensor.shape, dtype=torch.float32).normal_(0.0, std, generator=gen)
                tensor.copy_(draw.to(tensor.dtype))
    return model


def build_random_llama(
    config: "LlamaConfig", seed: int, std: float = 0.02, dtype: torch.dtype = torch.float32, device="cpu"
) -> "Llama3_2":
    """Allocate without default init, fill with :func:`init_random_weights_`, move to device."""
    with torch.device("meta"):
        model = Llama3_2(config)
    model = model.to_empty(device="cpu")
    if config.tie_word_embeddings:
        model.lm_head.weight = model.embed.weight
    init_random_weights_(model, seed, std)
    return model.to(dtype=dtype, device=device).eval()


class _DecodeGraph:
    """A captured decode-only step (every request has one query token) for a fixed batch.

    The plan (table rows, contexts, query lengths) and token ids live in
    static device buffers that are refreshed before each replay; the packing
    kernel, all layers and the lm_head run inside the graph.  A graph is tied
    to one cache and one block-table tensor (the table is reallocated when it
    grows, which retires the graph).
    """

    def __init__(self, model: "Llama3_2", cache: PagedKVCache, batch: int) -> None:
        dev = cache.device
        self.batch = batch
        # the graph bakes in raw pointers: keep every buffer it touches alive
        self.model = model
        self.workspace = ops.decode_workspace(dev, batch, model.config.q_head_num, model.config.head_dim)
        self.ids = torch.zeros(batch, dtype=torch.long, device=dev)
        self.plan = torch.zeros((3, batch), dtype=torch.int32, device=dev)
        self.table = cache.device_block_tables()
        self.generation = model._ensure_fused()
        self.graph = torch.cuda.CUDAGraph()
        launches = ops.LAUNCHES
        with torch.cuda.graph(self.graph):
            meta = ops.pack_ragged(
                self.plan,
                batch,
                self.table,
                cache.block_size,
                cache.allocator.num_blocks,
                num_decode=batch,
                max_query_len=1,
            )
            self.logits = model.run_ragged(self.ids, meta, cache)
        # library kernels inside the graph, counted again at every replay
        self.kernels = ops.LAUNCHES - launches
        ops.LAUNCHES = launches

    def run(self, input_ids: torch.Tensor, plan_host: torch.Tensor) -> torch.Tensor:
        self.plan.copy_(plan_host.pin_memory(), non_blocking=True)
        self.ids.copy_(input_ids)
        self.graph.replay()
        ops._count(self.kernels)
        return self.logits.clone()


class Llama3_2(nn.Module):
    """Reference models/llama.py:95-394 module tree and entry points."""

    # Replay decode-only steps from captured CUDA graphs (one per batch size).
    cuda_graphs: bool = True
    # Run the decoder layers of a ragged step through the C++ layer loop when
    # it is built (the Python loop issues the same kernels, with more host time).
    native_layer_loop: bool = True

    def __init__(self, config: LlamaConfig) -> None:
        super().__init__()
        self.config = config
        self.embed = nn.Embedding(config.vocab_size, config.hidden_size)
        self.rope = build_rope(config)
        self.decoders = nn.ModuleList(
            [
                Llama3Decoder(
                    config.norm_eps,
                    config.q_head_num,
                    config.kv_head_num,
                    config.hidden_size,
                    config.mlp_inner_size,
                    self.rope,
                )
                for _ in range(config.num_layers)
            ]
        )
        self.final_rms = RmsNorm(config.hidden_size, config.norm_eps)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.embed.weight

    # ------------------------------------------------------------ core step
    def run_ragged(
        self,
        input_ids: torch.Tensor,
        meta: ops.RaggedMeta,
        cache: PagedKVCache,
        *,
        rope_positions: torch.Tensor | None = None,
        logit_rows: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Embed -> decoders -> norm -> lm_head over flattened tokens.

        Residual adds are folded into the next RMSNorm (fused kernel), so a
        layer is: add+norm, q/k/v GEMMs, RoPE+KV write, attention, o_proj,
        add+norm, gate/up GEMMs, SiLU*up, down GEMM.
        """
        self._ensure_fused()
        table = self.embed.weight
        x = ops.embed_rows(input_ids, table) if ops.embed_eligible(table) else self.embed(input_ids)
        positions = meta.positions if rope_positions is None else rope_positions
        sin, cos = self.rope.sin_cos(positions, x.dtype)
        ext = ops.layer_loop_ext() if (self.native_layer_loop and x.is_cuda) else None
        layer_args = self._layer_loop_args(x.dtype) if ext is not None else None
        if layer_args is not None:
            normed = self._run_layers_native(ext, layer_args, x, meta, cache, sin, cos, logit_rows)
            return self.lm_head(normed)
        first = self.decoders[0].pre_norm
        residual = x
        _, normed = ops.add_rmsnorm(x, None, first.weight, first.eps)
        last = len(self.decoders) - 1
        for layer_index, decoder in enumerate(self.decoders):
            mlp_out, h = decoder.step(normed, residual, meta, cache, layer_index, sin, cos)
            if layer_index < last:
                nxt = self.decoders[layer_index + 1].pre_norm
                residual, normed = ops.add_rmsnorm(mlp_out, h, nxt.weight, nxt.eps)
            else:
                if logit_rows is not None:
                    mlp_out = mlp_out.index_select(0, logit_rows)
                    h = h.index_select(0, logit_rows)
                _, normed = ops.add_rmsnorm(mlp_out, h, self.final_rms.weight, self.final_rms.eps, want_sum=False)
        return self.lm_head(normed)

    def _layer_loop_args(self, dtype: torch.dtype) -> tuple[list[torch.Tensor], list[float]] | None:
        """Per-layer weights for the C++ layer loop, or None where the Python loop must run.

        Rebuilt every step from the module dictionaries, with the same checks
        as the Python loop: fused q/k/v and gate/up buffers still back the
        projection weights, no forward hooks on o_proj / down_proj (or global
        ones) and no biases, so both loops compute the same thing.
        """
        hooks = nn.modules.module
        if hooks._global_forward_hooks or hooks._global_forward_pre_hooks:
            return None
        weights: list[torch.Tensor] = []
        eps: list[float] = []
        for decoder in self.decoders:
            mods = decoder.__dict__["_modules"]
            attn, ffn = mods["attn"], mods["ffn"]
            qkv = fused_weight(attn, ("q_proj", "k_proj", "v_proj"), "_qkv")
            gate_up = fused_weight(ffn, ("gate_proj", "up_proj"), "_gate_up")
            if qkv is None or gate_up is None or qkv.dtype != dtype:
                return None
            o_proj, down = attn.__dict__["_modules"]["o_proj"], ffn.__dict__["_modules"]["down_proj"]
            if o_proj._forward_hooks or o_proj._forward_pre_hooks or down._forward_hooks or down._forward_pre_hooks:
                return None
            o_params, down_params = o_proj._parameters, down._parameters
            if o_params["bias"] is not None or down_params["bias"] is not None:
                return None
            pre, post = mods["pre_norm"], mods["post_norm"]
            weights += (pre._parameters["weight"], qkv, o_params["weight"], post._parameters["weight"], gate_up,
                        down_params["weight"])
            eps += (pre.eps, post.eps)
        return weights, eps

    def _run_layers_native(self, ext, layer_args, x, meta, cache, sin, cos, logit_rows) -> torch.Tensor:
        """All decoder layers and the final norm through the C++ layer loop."""
        weights, eps = layer_args
        attn = self.decoders[0].attn
        hq, h, d = attn.q_head_num, attn.kv_head_num, attn.head_dim
        keys = cache.keys
        device = x.device
        dec_ws = ops.decode_workspace(device, max(meta.num_decode, 1), hq, d)
        var_ws = None
        if meta.num_prefill:
            need = int(ops.lib.nie_varlen_workspace_size(meta.num_prefill, meta.max_query_len, meta.max_seq_len, hq))
            var_ws = ops.varlen_workspace(device, need) if need else None
        normed, launches = ext.run_layers(
            x, weights, eps, self.final_rms.weight, self.final_rms.eps,
            meta.slot_mapping, meta.block_tables, meta.seq_lens, meta.query_start_loc, meta.table_rows,
            meta.decode_list, meta.prefill_list, meta.num_decode, meta.num_prefill, meta.max_query_len,
            meta.max_seq_len, logit_rows, keys, cache.values, sin, cos, hq, h, d, self.decoders[0].ffn.inner_size,
            dec_ws, ops.decode_launch_count(keys.dtype, keys.shape[2], h, d, hq), var_ws,
            ops.STREAM_LINEAR, ops.error_flag(device),
        )
        ops._count(launches)
        return normed

    def _ensure_fused(self) -> int:
        """Keep q/k/v and gate/up weights in single buffers; returns their generation.

        A cheap signature (first and last layer pointers) detects parameters
        replaced wholesale, e.g. by ``.to()``; the buffers are then rebuilt and
        the generation bumps, which retires captured graphs.
        """
        first, last = self.decoders[0], self.decoders[-1]
        sig = (first.attn.q_proj.weight.data_ptr(), last.ffn.up_proj.weight.data_ptr())
        if self.__dict__.get("_fused_sig") != sig:
            changed = False
            for decoder in self.decoders:
                changed = decoder.fuse_projections() or changed
            if changed:
                self.__dict__["_weights_gen"] = self.__dict__.get("_weights_gen", 0) + 1
            self.__dict__["_fused_sig"] = (first.attn.q_proj.weight.data_ptr(), last.ffn.up_proj.weight.data_ptr())
        return self.__dict__.get("_weights_gen", 0)

    def capture_decode_graphs(self, cache: PagedKVCache, batches) -> int:
        """Capture the decode-step graphs of the given batch sizes ahead of use.

        A batch size seen for the first time otherwise runs eagerly and is
        captured on the spot, stalling every request of that step.  Call after
        at least one step has run on this model (library handles and fused
        weights exist), with the cache's block table already sized by
        ``PagedKVCache.reserve_table`` (growing it retires the graphs).
        Returns the number of graphs captured.
        """
        table = cache.device_block_tables()
        graphs = cache.__dict__.setdefault("_decode_graphs", {})
        generation = self._ensure_fused()
        made = 0
        for batch in batches:
            key = (id(self), batch)
            graph = graphs.get(key)
            if graph is not None and graph.table is table and graph.generation == generation:
                continue
            graphs[key] = _DecodeGraph(self, cache, batch)
            made += 1
        return made

    def _decode_step(
        self,
        input_ids: torch.Tensor,
        cache: PagedKVCache,
        sequence_ids: tuple[str, ...],
        context_lengths: tuple[int, ...],
    ) -> torch.Tensor:
        """One decode-only step ([R] ids -> [R, vocab] logits), replayed from a CUDA graph.

        The first step of a given batch size runs eagerly (it doubles as the
        warm-up) and then captures the graph used by later steps.  Graphs are
        stored on the cache, so they die with it.
        """
        batch = len(sequence_ids)
        table = cache.device_block_tables()
        graphs = cache.__dict__.setdefault("_decode_graphs", {})
        key = (id(self), batch)
        generation = self._ensure_fused()
        graph = graphs.get(key)
        if graph is not None and (graph.table is not table or graph.generation != generation):
            graph = None  # the block-table tensor or the weight buffers were reallocated
        if graph is None:
            meta = cache.pack(sequence_ids, context_lengths, (1,) * batch)
            logits = self.run_ragged(input_ids, meta, cache)
            graphs[key] = _DecodeGraph(self, cache, batch)
            return logits
        rows = [cache.table_row(s) for s in sequence_ids]
        plan = torch.tensor([rows, list(context_lengths), [1] * batch], dtype=torch.int32)
        return graph.run(input_ids, plan)

    def _use_graph(self, cache: PagedKVCache, query_lengths) -> bool:
        return (
            self.cuda_graphs
            and cache.device.type == "cuda"
            and all(q == 1 for q in query_lengths)
            and not torch.cuda.is_current_stream_capturing()
        )

    # -------------------------------------------------------- ragged entry
    def forward_ragged(
        self,
        input_ids: torch.Tensor,
        *,
        kv_cache: PagedKVCache,
        sequence_ids: tuple[str, ...],
        query_start_loc: torch.Tensor,
    ) -> torch.Tensor:
        """Flattened variable-query step (reference llama.py:339-394)."""
        if input_ids.ndim != 1 or input_ids.numel() == 0:
            raise ValueError("input_ids must be a non-empty 1D tensor")
        if not isinstance(kv_cache, PagedKVCache):
            raise TypeError("kv_cache must be a PagedKVCache")
        if not sequence_ids or len(set(sequence_ids)) != len(sequence_ids):
            raise ValueError("sequence_ids must be non-empty and unique")
        if query_start_loc.ndim != 1 or query_start_loc.numel() != len(sequence_ids) + 1:
            raise ValueError("query_start_loc must have one boundary per sequence")
        if query_start_loc.device != input_ids.device:
            raise ValueError("query_start_loc must be on the input device")
        boundaries = getattr(query_start_loc, HOST_BOUNDARIES, None)
        if boundaries is None:
            boundaries = query_start_loc.tolist()
        if boundaries[0] != 0 or boundaries[-1] != input_ids.numel():
            raise ValueError("query_start_loc must span all input tokens")
        if any(end <= start for start, end in zip(boundaries, boundaries[1:])):
            raise ValueError("each ragged query must contain at least one token")

        context_lengths = tuple(kv_cache.get_sequence_length(s) for s in sequence_ids)
        query_lengths = tuple(b - a for a, b in zip(boundaries, boundaries[1:]))
        for s, c, q in zip(sequence_ids, context_lengths, query_lengths):
            if c + q > self.config.max_seq_len:
                raise ValueError(f"Sequence length {c + q} exceeds max_seq_len={self.config.max_seq_len}")
            kv_cache.ensure_capacity(s, c + q)

        last_only = bool(getattr(query_start_loc, LAST_ROWS_ONLY, False))
        if self._use_graph(kv_cache, query_lengths):
            # every row is its request's last row: full and last-row logits coincide
            logits = self._decode_step(input_ids, kv_cache, tuple(sequence_ids), context_lengths)
        else:
            meta = kv_cache.pack(tuple(sequence_ids), context_lengths, query_lengths)
            logits = self.run_ragged(
                input_ids, meta, kv_cache, logit_rows=meta.last_token_index if last_only else None
            )
        for s, q in zip(sequence_ids, query_lengths):
            kv_cache.advance(s, q)
        if last_only:
            setattr(logits, LAST_ROWS_DONE, True)
        return logits

    # ------------------------------------------------------- batched entry
    def forward(
        self,
        x: torch.Tensor,
        kv_cache: PagedKVCache | None = None,
        attention_mask: torch.Tensor | None = None,
        position_ids: torch.Tensor | None = None,
        sequence_id: str = "default",
        sequence_ids: tuple[str, ...] | None = None,
    ) -> torch.Tensor:
        """Batched paged decode / equal-length paged prefill (reference llama.py:127-337).

        ``kv_cache=None`` runs a causal prefill through a temporary paged
        cache (no padding masks).  The reference's contiguous ``KVCache`` and
        left-padded dense paths are not part of this build.
        """
        if kv_cache is None:
            return self._forward_uncached(x, attention_mask, position_ids)
        if not isinstance(kv_cache, PagedKVCache):
            raise NotImplementedError("only PagedKVCache is supported by nano_infer_engine_b200")
        batch, seq_len = x.shape[0], x.shape[1]
        decode = seq_len == 1
        if sequence_ids is None:
            if batch != 1:
                raise ValueError("sequence_ids is required for batched paged inference")
            ids: tuple[str, ...] = (sequence_id,)
        else:
            if not isinstance(sequence_ids, tuple):
                raise TypeError("sequence_ids must be a tuple")
            if len(sequence_ids) != batch:
                raise ValueError("sequence_ids must match the batch size")
            if any(not isinstance(s, str) or not s for s in sequence_ids):
                raise ValueError("sequence IDs must be non-empty strings")
            if len(set(sequence_ids)) != len(sequence_ids):
                raise ValueError("sequence IDs must be unique within a batch")
            ids = sequence_ids
        lengths = tuple(kv_cache.get_sequence_length(s) for s in ids)
        if not decode and len(set(lengths)) != 1:
            raise ValueError("batched paged prefill currently requires equal sequence lengths")
        kv_position = lengths[0]
        total = max(lengths) + 1 if decode else kv_position + seq_len
        if total > self.config.max_seq_len:
            raise ValueError(f"Sequence length {total} exceeds max_seq_len={self.config.max_seq_len}")
        for s, n in zip(ids, lengths):
            kv_cache.ensure_capacity(s, n + 1 if decode else total)

        if decode:
            if attention_mask is not None:
                if attention_mask.device != x.device:
                    raise ValueError("attention_mask must be on the same device as x")
                if not bool(attention_mask.all()):
                    raise ValueError("paged inference does not support padding masks")
            if position_ids is not None:
                if position_ids.shape != (batch, 1):
                    raise ValueError(
                        f"position_ids must have shape {(batch, 1)}, got {tuple(position_ids.shape)}"
                    )
                if position_ids.device != x.device:
                    raise ValueError("position_ids must be on the same device as x")
                expected = torch.tensor(lengths, dtype=torch.long, device=x.device)[:, None]
                if not torch.equal(position_ids, expected):
                    raise ValueError("position_ids must match paged cache sequence lengths")
            rope_positions = None
        else:
            if attention_mask is not None:
                if attention_mask.shape != (batch, total):
                    raise ValueError(
                        f"attention_mask must have shape {(batch, total)}, got {tuple(attention_mask.shape)}"
                    )
                if attention_mask.device != x.device:
                    raise ValueError("attention_mask must be on the same device as x")
                if not bool(attention_mask.bool().all()):
                    raise ValueError("paged inference does not support padding masks")
            rope_positions = None
            if position_ids is not None:
                if position_ids.shape != (batch, seq_len):
                    raise ValueError(
                        f"position_ids must have shape {(batch, seq_len)}, got {tuple(position_ids.shape)}"
                    )
                if position_ids.device != x.device:
                    raise ValueError("position_ids must be on the same device as x")
                rope_positions = position_ids.reshape(-1)

        if decode and position_ids is None and self._use_graph(kv_cache, (1,) * batch):
            logits = self._decode_step(x.reshape(-1), kv_cache, ids, lengths)
            for s in ids:
                kv_cache.advance(s, 1)
            return logits.view(batch, 1, -1)
        meta = kv_cache.pack(ids, lengths, (seq_len,) * batch)
        last_only = bool(getattr(x, LAST_ROWS_ONLY, False))
        logits = self.run_ragged(
            x.reshape(-1),
            meta,
            kv_cache,
            rope_positions=rope_positions,
            logit_rows=meta.last_token_index if last_only else None,
        )
        for s in ids:
            kv_cache.advance(s, seq_len)
        if last_only:
            return logits.view(batch, 1, -1)
        return logits.view(batch, seq_len, -1)

    def _forward_uncached(self, x, attention_mask, position_ids) -> torch.Tensor:
        if attention_mask is not None and not bool(attention_mask.bool().all()):
            raise NotImplementedError("padding masks (left-padded dense batches) are not supported")
        batch, seq_len = x.shape[0], x.shape[1]
        if seq_len > self.config.max_seq_len:
            raise ValueError(f"Sequence length {seq_len} exceeds max_seq_len={self.config.max_seq_len}")
        block_size = 16
        blocks = batch * (-(-seq_len // block_size))
        cache = PagedKVCache(
            blocks,
            block_size,
            self.config.num_layers,
            self.config.kv_head_num,
            self.config.head_dim,
            self.embed.weight.dtype,
            x.device,
        )
        ids = tuple(f"__uncached_{i}" for i in range(batch))
        return self.forward(x, kv_cache=cache, position_ids=position_ids, sequence_ids=ids)
