"""Tensor-parallel Llama graphs: one rank's share of prefill and batched decode.

The reference (chomikgrad/llama.py) is single-device.  Here each of
``size`` ranks holds:

* a contiguous block of query heads (``heads = H / size``) with the matching
  rows of q_proj and columns of o_proj;
* the KV heads those queries read: ``num_key_value_heads / size`` heads each,
  or, with more ranks than KV heads, the one KV head of its query block
  (replicated on ``size / num_key_value_heads`` ranks);
* ``intermediate_size / size`` rows of gate_proj and up_proj and the matching
  columns of down_proj;
* everything else (embedding, norms) whole, and the lm_head whole or, with
  ``vocab_shard``, ``vocab_size / size`` of its rows.

The rank's graph is the reference's graph over those shards, with one
change: the O and down projections produce partial sums, which
``all_reduce`` adds up over the group before the residual add.  The
all-reduce is an identity node (``x * 1``) carrying an ``all_reduce``
lowering hint, the same mechanism as the reference's preferred lowerings
(llama.py:13-25): on one rank the portable graph is exact, and the
``cuda-b200`` planner lowers the hint to an NCCL all-reduce step of the
compiled program (``cuda_b200.parallel``).  A vocabulary-sharded lm_head
produces this rank's columns of the logits.  The prefill gathers them
(``all_gather``: the portable form ``x.reshape(1, ...) * ones(G, 1, ...)``,
exact on one rank, with an ``all_gather`` hint lowered to NCCL's
all-gather), so its program returns the whole logits.  The batched decode
step returns this rank's columns only, and the greedy token of every row
comes from a distributed argmax (``cb_argmax_rows_sharded``: each rank's
(value, global index) winner per row, all-gathered, the same pick on every
rank -- np.argmax's order over the whole row), so a step exchanges 16 bytes
per row and rank instead of the logits, while each rank reads 1/size of the
lm_head.

Per rank and step the decode reads 1/size of the sharded weights (plus the
replicated ones) and exchanges 2 x layers x batch x hidden float32 values.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from chomikgrad.llama import LlamaConfig, LlamaForCausalLM, _prefer_lowering, _rope_rotations, position_selector
from chomikgrad.tensor import Tensor, compile_graph, no_grad

from .batched import BatchedDecoderStep, BatchedPrefill, BatchedRuntime
from .graphs import MASKED, GraphHelpers


@dataclass(frozen=True)
class ShardLayout:
    """What rank ``rank`` of ``size`` holds (row/column ranges of the HF weights)."""

    size: int
    rank: int
    heads: int          # query heads on this rank
    kv_heads: int       # KV heads on this rank
    head_size: int
    intermediate: int   # gate/up rows on this rank
    q_start: int        # first q_proj row (= first o_proj column)
    kv_start: int       # first k_proj / v_proj row
    i_start: int        # first gate/up row (= first down_proj column)
    vocab: int = 0      # lm_head rows on this rank (vocab_shard); 0: the whole lm_head
    vocab_start: int = 0

    @property
    def vocab_shard(self) -> bool:
        return self.vocab > 0

    @property
    def vocab_rows(self) -> slice:
        return slice(self.vocab_start, self.vocab_start + self.vocab)

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    @property
    def q_rows(self) -> slice:
        return slice(self.q_start, self.q_start + self.heads * self.head_size)

    @property
    def kv_rows(self) -> slice:
        return slice(self.kv_start, self.kv_start + self.kv_heads * self.head_size)

    @property
    def i_rows(self) -> slice:
        return slice(self.i_start, self.i_start + self.intermediate)


def shard_layout(config: LlamaConfig, size: int, rank: int, *, vocab_shard: bool = False) -> ShardLayout:
    if size < 1 or not 0 <= rank < size:
        raise ValueError(f"rank {rank} of {size}")
    if vocab_shard and config.vocab_size % size:
        raise ValueError(f"{size} ranks must divide the vocabulary of {config.vocab_size} to shard the lm_head")
    vocab = config.vocab_size // size if vocab_shard else 0
    nh, nkv, hd = config.num_attention_heads, config.num_key_value_heads, config.head_size
    if nh % size or config.intermediate_size % size:
        raise ValueError(f"{size} ranks must divide the {nh} heads and the intermediate size "
                         f"{config.intermediate_size}")
    heads = nh // size
    if size <= nkv:
        if nkv % size:
            raise ValueError(f"{size} ranks must divide the {nkv} KV heads")
        kv_heads = nkv // size
        kv_first = rank * kv_heads
    else:
        if size % nkv:
            raise ValueError(f"{size} ranks must be a multiple of the {nkv} KV heads")
        kv_heads = 1
        kv_first = (rank * heads) // config.query_groups
    inter = config.intermediate_size // size
    return ShardLayout(size=size, rank=rank, heads=heads, kv_heads=kv_heads, head_size=hd,
                       intermediate=inter, q_start=rank * heads * hd, kv_start=kv_first * hd,
                       i_start=rank * inter, vocab=vocab, vocab_start=rank * vocab)


def _contiguous(value):
    if hasattr(value, "contiguous"):  # torch
        return value.contiguous()
    return np.ascontiguousarray(value)


def shard_weights(config: LlamaConfig, weights: Mapping[str, Any], layout: ShardLayout) -> Dict[str, Any]:
    """This rank's weights (same names; NumPy or torch arrays, sliced and made contiguous)."""
    out: Dict[str, Any] = {}
    for name, w in weights.items():
        if name.endswith("q_proj.weight"):
            out[name] = _contiguous(w[layout.q_rows])
        elif name.endswith(("k_proj.weight", "v_proj.weight")):
            out[name] = _contiguous(w[layout.kv_rows])
        elif name.endswith("o_proj.weight"):
            out[name] = _contiguous(w[:, layout.q_rows])
        elif name.endswith(("gate_proj.weight", "up_proj.weight")):
            out[name] = _contiguous(w[layout.i_rows])
        elif name.endswith("down_proj.weight"):
            out[name] = _contiguous(w[:, layout.i_rows])
        elif name == "lm_head.weight" and layout.vocab_shard:
            out[name] = _contiguous(w[layout.vocab_rows])
        else:
            out[name] = w
    return out


def all_reduce(partial: Tensor, group: str) -> Tensor:
    """Sum of ``partial`` over the ranks of ``group``; on one rank the graph is ``partial`` itself."""
    return _prefer_lowering(partial * 1, "all_reduce", (partial,), group)


def all_gather(part: Tensor, group: str, size: int, dtype) -> Tensor:
    """(size, *part.shape): every rank's ``part`` in rank order; on one rank the graph is exact."""
    spread = part.reshape(1, *part.shape) * Tensor.ones((size,) + (1,) * len(part.shape), dtype=dtype)
    return _prefer_lowering(spread, "all_gather", (part,), group)


class _ShardMixin(GraphHelpers):
    """Shared overrides of the reference's building blocks: local head counts in the GQA
    broadcast, the MLP all-reduce, the vocabulary-sharded lm_head."""

    layout: ShardLayout
    group_name: str
    gather_logits = True  # a vocabulary-sharded lm_head returns the whole logits (else this rank's columns)

    def _init_shard(self, layout: ShardLayout, group: str) -> None:
        self.layout = layout
        self.group_name = group
        self.kv_repeat = Tensor.ones((1, 1, layout.group, 1, 1), dtype=self.dtype)

    def _repeat_kv(self, inputs: Tensor) -> Tensor:
        b, kv, t, d = inputs.shape
        spread = inputs.reshape(b, kv, 1, t, d) * self.kv_repeat
        return spread.reshape(b, self.layout.heads, t, d)

    def _reduce(self, partial: Tensor) -> Tensor:
        """The group's sum of a row-sharded projection (nothing to add on one rank)."""
        return partial if self.layout.size == 1 else all_reduce(partial, self.group_name)

    def _mlp(self, inputs: Tensor, layer: int) -> Tensor:
        return self._reduce(LlamaForCausalLM._mlp(self, inputs, layer))

    def _linear(self, inputs: Tensor, weight: Tensor) -> Tensor:
        """``x @ W.T``; through a vocabulary-sharded lm_head, the whole logits gathered from the group
        (or, with ``gather_logits`` off, this rank's columns)."""
        out = inputs @ weight.T
        if self.layout.vocab_shard and self.gather_logits and weight is self.weights.get("lm_head.weight"):
            rows, cols = out.shape
            gathered = all_gather(out, self.group_name, self.layout.size, self.dtype)  # (G, rows, V / G)
            return gathered.permute(1, 0, 2).reshape(rows, self.layout.size * cols)
        return out


def _init_model(model, config: LlamaConfig, weights: Mapping[str, Tensor], *, sequence_length: int,
                dtype, cache_length: Optional[int]) -> None:
    """LlamaForCausalLM's fields without its whole-model shape check (the weights are shards)."""
    config.validate()
    model.config = config
    model.weights = dict(weights)
    model.sequence_length = sequence_length
    model.dtype = np.dtype(dtype)
    model.cache_length = cache_length
    model.cache_placement = None
    if cache_length is not None:
        place = np.zeros((sequence_length, cache_length), dtype=model.dtype)
        place[np.arange(sequence_length), np.arange(sequence_length)] = 1
        model.cache_placement = Tensor(place)
    mask = np.triu(np.full((sequence_length, sequence_length), MASKED, dtype=model.dtype), k=1)
    model.causal_mask = Tensor(mask.reshape(1, 1, sequence_length, sequence_length))
    model.rotations = Tensor(_rope_rotations(sequence_length, config.head_size, config.rope_theta, model.dtype))


class TensorParallelPrefill(_ShardMixin, LlamaForCausalLM):
    """One rank's prefill (llama.py:382-433) over its shards, all-reducing O and down.

    The reference's ``_forward`` runs unchanged; this class replaces its
    ``_attention`` (local head counts, all-reduced O projection), ``_mlp``
    and ``_linear`` (see ``_ShardMixin``).
    """

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], layout: ShardLayout, *,
                 sequence_length: int, dtype, cache_length: int, group: str = "tp") -> None:
        _init_model(self, config, weights, sequence_length=sequence_length, dtype=dtype,
                    cache_length=cache_length)
        self._init_shard(layout, group)

    def _attention(self, inputs: Tensor, layer: int) -> Tuple[Tensor, Tensor, Tensor]:
        lay = self.layout
        p = f"model.layers.{layer}.self_attn"
        batch, tokens, _ = inputs.shape
        query = self._linear(inputs, self.weights[f"{p}.q_proj.weight"])
        key = self._linear(inputs, self.weights[f"{p}.k_proj.weight"])
        value = self._linear(inputs, self.weights[f"{p}.v_proj.weight"])
        query = query.reshape(batch, tokens, lay.heads, lay.head_size).permute(0, 2, 1, 3)
        key = key.reshape(batch, tokens, lay.kv_heads, lay.head_size).permute(0, 2, 1, 3)
        value = value.reshape(batch, tokens, lay.kv_heads, lay.head_size).permute(0, 2, 1, 3)
        query = self._apply_rope(query)
        key = self._apply_rope(key)
        attended = self._attend(query, key, value, self.causal_mask)
        merged = attended.permute(0, 2, 1, 3).reshape(batch, tokens, lay.heads * lay.head_size)
        partial = self._linear(merged, self.weights[f"{p}.o_proj.weight"])
        return self._reduce(partial), key, value


class TensorParallelBatchedPrefill(TensorParallelPrefill):
    """B prompts of equal length through one rank's prefill as one graph: the forward of
    ``BatchedPrefill`` over this rank's shards (every Linear one (B*T)-row GEMM)."""

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], layout: ShardLayout, *, batch: int,
                 sequence_length: int, dtype, cache_length: int, group: str = "tp") -> None:
        super().__init__(config, weights, layout, sequence_length=sequence_length, dtype=dtype,
                         cache_length=cache_length, group=group)
        if batch <= 0:
            raise ValueError("batch must be positive")
        self.batch = batch

    _forward = BatchedPrefill._forward


class TensorParallelDecoderStep(_ShardMixin, BatchedDecoderStep):
    """One rank's batched decode step over its shards; caches are (B, kv_heads, ctx, hd) per rank.

    With a vocabulary-sharded lm_head the logits are this rank's (B, vocab / size) columns."""

    gather_logits = False

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], layout: ShardLayout, *,
                 batch: int, cache_length: int, dtype, group: str = "tp") -> None:
        if batch <= 0:
            raise ValueError("batch must be positive")
        if not 0 < cache_length <= config.max_position_embeddings:
            raise ValueError("invalid KV cache length")
        _init_model(self, config, weights, sequence_length=1, dtype=dtype, cache_length=None)
        self.cache_length = cache_length
        self.batch = batch
        self._init_shard(layout, group)

    def __call__(self, token_matrix: Tensor, rotation: Tensor, attention_mask: Tensor,
                 write_mask: Tensor, caches: Sequence[Tuple[Tensor, Tensor]], *,
                 position: Optional[Tensor] = None) -> Tuple[Tensor, ...]:
        c, ctx, b, lay = self.config, self.cache_length, self.batch, self.layout
        hd = lay.head_size
        if token_matrix.shape != (b, 1):
            raise ValueError(f"batched decode takes ({b}, 1) token ids")
        if len(caches) != c.num_hidden_layers:
            raise ValueError("decode requires one KV cache pair per layer")
        hidden = self._embed(token_matrix)  # (B, 1, H)
        updated = []
        cache_shape = (b, lay.kv_heads, ctx, hd)
        for layer, (old_key, old_value) in enumerate(caches):
            if old_key.shape != cache_shape or old_value.shape != cache_shape:
                raise ValueError("KV cache shard has the wrong shape")
            p = f"model.layers.{layer}"
            a = f"{p}.self_attn"
            normed = self._rms_norm(hidden, self.weights[f"{p}.input_layernorm.weight"])
            query = self._linear(normed, self.weights[f"{a}.q_proj.weight"]).reshape(b, lay.heads, 1, hd)
            key = self._linear(normed, self.weights[f"{a}.k_proj.weight"]).reshape(b, lay.kv_heads, 1, hd)
            value = self._linear(normed, self.weights[f"{a}.v_proj.weight"]).reshape(b, lay.kv_heads, 1, hd)
            query = self._apply_rotation(query, rotation, position)
            key = self._apply_rotation(key, rotation, position)
            new_key = old_key * (1 - write_mask) + key * write_mask
            new_value = old_value * (1 - write_mask) + value * write_mask
            updated.extend((new_key, new_value))
            attended = self._attend(query, new_key, new_value, attention_mask)
            merged = attended.permute(0, 2, 1, 3).reshape(b, 1, lay.heads * hd)
            partial = self._linear(merged, self.weights[f"{a}.o_proj.weight"])
            hidden = hidden + self._reduce(partial)
            normed = self._rms_norm(hidden, self.weights[f"{p}.post_attention_layernorm.weight"])
            hidden = hidden + self._mlp(normed, layer)
        hidden = self._rms_norm(hidden, self.weights["model.norm.weight"])
        logits = self._linear(hidden.reshape(b, c.hidden_size), self.weights["lm_head.weight"])
        return (logits, *updated)


class TensorParallelRuntime(BatchedRuntime):
    """Prefill and batched greedy decode of one rank of a tensor-parallel group.

    ``weights`` are this rank's shards (``shard_weights``).  Every rank runs
    the same calls with the same token ids; the greedy tokens are the same on
    every rank.  With a replicated lm_head ``decode_batch`` returns the whole
    logits; with a vocabulary-sharded one it returns this rank's columns,
    ``greedy_rows`` picks the tokens by the distributed argmax and
    ``full_logits`` gathers whole rows (collective: every rank calls it).
    """

    def __init__(self, config: LlamaConfig, weights, layout: ShardLayout, *, batch: int,
                 compiler: str = "cuda-b200", dtype=None, group: str = "tp") -> None:
        super().__init__(config, weights, batch=batch, compiler=compiler, dtype=dtype)
        self.layout = layout
        self.group = group
        self._argmax_scratch = None
        self._argmax_out = None

    def _comm_handle(self) -> Optional[int]:
        from . import parallel

        return parallel.get_group(self.group).handle if self.layout.size > 1 else None

    def _argmax_rows(self, program, logits_view, out_ptr: int, stream: int) -> None:
        if not self.layout.vocab_shard:
            super()._argmax_rows(program, logits_view, out_ptr, stream)
            return
        self._sharded_argmax(program.ptr(logits_view), logits_view.dtype, logits_view.shape[-1], out_ptr, stream)

    def _sharded_argmax(self, ptr: int, dtype, width: int, out_ptr: int, stream: int) -> None:
        import torch

        from . import _lib

        if self._argmax_scratch is None:  # (size + 1) * batch 16-byte records
            self._argmax_scratch = torch.empty((self.layout.size + 1) * self.batch * 4, dtype=torch.float32,
                                               device=self.device.torch_device)
        _lib.call("cb_argmax_rows_sharded", self._comm_handle(), self.layout.size, ptr, _lib.dtype_code(dtype),
                  self.batch, width, self.layout.vocab_start, self._argmax_scratch.data_ptr(), out_ptr, stream)

    def greedy_rows(self, logits) -> List[int]:
        if not self.layout.vocab_shard:
            return super().greedy_rows(logits)
        tensor = logits.tensor if hasattr(logits, "tensor") else logits
        self._sharded_argmax(tensor.data_ptr(), self.device.dtype(logits), logits.shape[-1],
                             self._ensure_out(), self.device.stream())
        return [int(t) for t in self._argmax_out.tolist()]

    def _ensure_out(self) -> int:
        import torch

        if self._argmax_out is None:
            self._argmax_out = torch.empty(self.batch, dtype=torch.int64, device=self.device.torch_device)
        return self._argmax_out.data_ptr()

    def full_logits(self, logits):
        """Whole (B, vocab) rows: this rank's columns all-gathered from the group (collective)."""
        if not self.layout.vocab_shard:
            return logits
        import torch

        from . import _lib

        tensor = logits.tensor if hasattr(logits, "tensor") else logits
        local = tensor.reshape(self.batch, -1).float().contiguous()
        size, cols = self.layout.size, local.shape[1]
        gathered = torch.empty((size, self.batch, cols), dtype=torch.float32, device=local.device)
        if size == 1:
            gathered[0].copy_(local)
        else:
            from . import parallel

            parallel.get_group(self.group).all_gather(local.data_ptr(), gathered.data_ptr(), local.numel(),
                                                      _lib.F32, self.device.stream())
        whole = gathered.permute(1, 0, 2).reshape(self.batch, size * cols)
        return self.device.array(whole)

    def prefill(self, prompt_ids: Sequence[int], context: int) -> Tuple[Any, List[Any]]:
        ids = np.asarray(prompt_ids, dtype=np.int32).reshape(1, -1)
        key = (ids.shape[1], context)
        cached = self._prefill.get(key)
        with no_grad():
            if cached is None:
                model = TensorParallelPrefill(self.config, self.weights, self.layout, sequence_length=ids.shape[1],
                                              dtype=self.dtype, cache_length=context, group=self.group)
                selector = position_selector(ids.shape[1] - 1, ids.shape[1], dtype=self.dtype)
                source = Tensor(ids, copy=False)
                outputs = model.prefill(source, Tensor(selector, copy=False))
                program = compile_graph(*outputs, compiler=self.compiler_name, dynamic_inputs=(source,))
                self._prefill[key] = (program, source._node)
                bindings = None
            else:
                program, node = cached
                bindings = {node: self.device.array(ids)}
            produced = program.run(bindings, synchronize=False)
        return produced[0], list(produced[1:])

    def prefill_batched(self, prompts: Sequence[Sequence[int]], context: int) -> Tuple[Any, List[Any]]:
        """The prompts through this rank's batched prefill program: the whole (B, vocab) logits
        and this rank's (B, kv_heads / G, context, head_size) caches."""
        ids = np.asarray(prompts, dtype=np.int32)
        if ids.ndim != 2 or ids.shape[0] == 0:
            raise ValueError("prompts must be a non-empty list of equal-length token lists")
        key = ("batched",) + ids.shape + (context,)
        cached = self._prefill.get(key)
        with no_grad():
            if cached is None:
                b, t = ids.shape
                model = TensorParallelBatchedPrefill(self.config, self.weights, self.layout, batch=b,
                                                     sequence_length=t, dtype=self.dtype, cache_length=context,
                                                     group=self.group)
                source = Tensor(ids, copy=False)
                outputs = model.prefill(source, Tensor(position_selector(t - 1, t, dtype=self.dtype), copy=False))
                program = compile_graph(*outputs, compiler=self.compiler_name, dynamic_inputs=(source,))
                self._prefill[key] = (program, source._node)
                bindings = None
            else:
                program, node = cached
                bindings = {node: self.device.array(ids)}
            produced = program.run(bindings, synchronize=False)
        return produced[0], list(produced[1:])

    def close(self) -> None:
        """Release every compiled program's CUDA graphs.

        The graphs hold the group's NCCL all-reduces; NCCL does not destroy
        a communicator that a live graph still uses, so close the runtime
        before ``parallel.destroy_group``.
        """
        for program, _ in list(self._prefill.values()) + list(self._batched.values()):
            program.close()
        self._prefill.clear()
        self._batched.clear()

    def batched_program(self, context: int, caches: List[Any], tokens: Sequence[int], position: int):
        cached = self._batched.get(context)
        if cached is not None:
            return cached
        host = self.batched_step_inputs(tokens, position, context)
        with no_grad():
            step = TensorParallelDecoderStep(self.config, self.weights, self.layout, batch=self.batch,
                                             cache_length=context, dtype=self.dtype, group=self.group)
            tensors = [Tensor(v, copy=False) for v in host]
            cache_tensors = [Tensor.from_native(v, backend=self.device.name, shape=tuple(v.shape),
                                                dtype=self.dtype) for v in caches]
            outputs = step(tensors[0], tensors[1], tensors[2], tensors[3],
                           list(zip(cache_tensors[::2], cache_tensors[1::2])), position=tensors[4])
            dynamic = [*tensors, *cache_tensors]
            program = compile_graph(*outputs, compiler=self.compiler_name, dynamic_inputs=dynamic)
        entry = (program, [t._node for t in dynamic])
        self._batched[context] = entry
        return entry
