"""Batched greedy decode of independent sequences (an extension of the plugin).

The reference's ``LlamaDecoderStep`` (chomikgrad/llama.py:436-543) takes one
token of one sequence.  ``BatchedDecoderStep`` builds the same six-op graph
for B sequences at once: every tensor gains a leading batch dimension, the
per-step RoPE rotation and masks are shared (the sequences advance in lock
step at the same position, as in the batched workloads: equal prompt
lengths), and each sequence reads and writes its own slice of the
(B, kv_heads, context, head_size) caches.  Per sequence the graph computes
exactly what ``LlamaDecoderStep`` computes; only the weight reads are shared,
which turns each Linear into a B-row matmul (the tcgen05 GEMM).

``BatchedRuntime`` prefills the prompts together (``BatchedPrefill``: the
reference's prefill, llama.py:432-433, with the batch dimension its layers
already carry), and then steps all sequences together, picking each next token by ``argmax_last_axis``
(chomikgrad/lazy.py:132-134; the reference's greedy sampler takes the first
maximum, generate_tinyllama.py:146-157).
"""

from __future__ import annotations

from typing import Any, List, Optional, Sequence, Tuple

import numpy as np

from chomikgrad.llama import LlamaConfig, LlamaDecoderStep, LlamaForCausalLM, _rope_rotations
from chomikgrad.tensor import Tensor, compile_graph, no_grad

from .device import DeviceArray
from .graphs import GraphHelpers, decode_masks
from .runtime import LlamaRuntime


class BatchedDecoderStep(GraphHelpers, LlamaDecoderStep):
    """One decode step of B independent sequences sharing the position.

    A subclass of the reference's ``LlamaDecoderStep``: the same validation
    of rotation, masks and caches, the same per-layer chain of the reference's
    own building blocks (``_rms_norm``, ``_linear``, ``_apply_rotation``,
    ``_repeat_kv``, ``_mlp``), with B in the leading dimension.
    """

    def __init__(self, config: LlamaConfig, weights, *, batch: int, cache_length: int,
                 dtype: np.dtype) -> None:
        super().__init__(config, weights, cache_length=cache_length, dtype=dtype)
        if batch <= 0:
            raise ValueError("batch must be positive")
        self.batch = batch

    def _check_step(self, token_matrix: Tensor, rotation: Tensor, attention_mask: Tensor,
                    write_mask: Tensor, caches, position: Optional[Tensor]) -> None:
        c, ctx, b = self.config, self.cache_length, self.batch
        if token_matrix.shape != (b, 1):
            raise ValueError(f"batched decode takes ({b}, 1) token ids")
        if rotation.shape != (1, 1, 1, c.head_size, c.head_size):
            raise ValueError("decode RoPE rotation has the wrong shape")
        if attention_mask.shape != (1, 1, 1, ctx) or write_mask.shape != (1, 1, ctx, 1):
            raise ValueError("decode masks have the wrong shape")
        if len(caches) != c.num_hidden_layers:
            raise ValueError("decode requires one KV cache pair per layer")
        if position is not None and position.shape != ():
            raise ValueError("decode position must be a scalar")

    def __call__(self, token_matrix: Tensor, rotation: Tensor, attention_mask: Tensor,
                 write_mask: Tensor, caches: Sequence[Tuple[Tensor, Tensor]], *,
                 position: Optional[Tensor] = None) -> Tuple[Tensor, ...]:
        self._check_step(token_matrix, rotation, attention_mask, write_mask, caches, position)
        c, ctx, b = self.config, self.cache_length, self.batch
        hd, nh, nkv = c.head_size, c.num_attention_heads, c.num_key_value_heads
        hidden = self._embed(token_matrix)  # (B, 1, H)
        updated = []
        for layer, (old_key, old_value) in enumerate(caches):
            if old_key.shape != (b, nkv, ctx, hd) or old_value.shape != (b, nkv, ctx, hd):
                raise ValueError("KV cache has the wrong shape")
            w = f"model.layers.{layer}"
            normed = self._rms_norm(hidden, self.weights[f"{w}.input_layernorm.weight"])
            q = self._linear(normed, self.weights[f"{w}.self_attn.q_proj.weight"]).reshape(b, nh, 1, hd)
            k = self._linear(normed, self.weights[f"{w}.self_attn.k_proj.weight"]).reshape(b, nkv, 1, hd)
            v = self._linear(normed, self.weights[f"{w}.self_attn.v_proj.weight"]).reshape(b, nkv, 1, hd)
            q = self._apply_rotation(q, rotation, position)
            k = self._apply_rotation(k, rotation, position)
            keys = old_key * (1 - write_mask) + k * write_mask
            values = old_value * (1 - write_mask) + v * write_mask
            updated.extend((keys, values))
            heads = self._attend(q, keys, values, attention_mask)
            hidden = hidden + self._linear(heads.permute(0, 2, 1, 3).reshape(b, 1, c.hidden_size),
                                           self.weights[f"{w}.self_attn.o_proj.weight"])
            normed = self._rms_norm(hidden, self.weights[f"{w}.post_attention_layernorm.weight"])
            hidden = hidden + self._mlp(normed, layer)
        hidden = self._rms_norm(hidden, self.weights["model.norm.weight"])
        logits = self._linear(hidden.reshape(b, c.hidden_size), self.weights["lm_head.weight"])
        return (logits, *updated)


class BatchedPrefill(GraphHelpers, LlamaForCausalLM):
    """The prefill of B prompts of equal length as one graph.

    The reference's ``LlamaForCausalLM`` checks for one prompt
    (llama.py:389-396) although its layers already carry a batch dimension
    (``_attention`` and ``_mlp`` take (batch, tokens, hidden)).  Here the
    token matrix is (B, T): every Linear becomes one (B*T)-row GEMM over the
    shared weights, the causal mask and the RoPE table broadcast over the
    batch, and each prompt's caches are placed as the reference places them
    (llama.py:411-418).  Per prompt the graph computes what the batch-1
    prefill computes.  Returns (B, vocab) logits of each prompt's last token
    and the (B, kv_heads, cache_length, head_size) caches.
    """

    def __init__(self, config: LlamaConfig, weights, *, batch: int, sequence_length: int, dtype: np.dtype,
                 cache_length: int) -> None:
        super().__init__(config, weights, sequence_length=sequence_length, dtype=dtype, cache_length=cache_length)
        if batch <= 0:
            raise ValueError("batch must be positive")
        self.batch = batch

    def _forward(self, token_matrix: Tensor, selector: Tensor, *, collect_cache: bool) -> Tuple[Tensor, ...]:
        c, b, t = self.config, self.batch, self.sequence_length
        if token_matrix.shape != (b, t):
            raise ValueError(f"batched prefill takes ({b}, {t}) token ids")
        if selector.shape != (1, t):
            raise ValueError("position selector has the wrong shape")
        hidden = self._embed(token_matrix)  # (B, T, H)
        caches = []
        for layer in range(c.num_hidden_layers):
            w = f"model.layers.{layer}"
            attended, key, value = self._attention(self._rms_norm(hidden, self.weights[f"{w}.input_layernorm.weight"]),
                                                   layer)
            hidden = hidden + attended
            if collect_cache:
                for part in (key, value):  # (B, kv, T, hd) -> (B, kv, ctx, hd) through the placement matrix
                    caches.append((part.permute(0, 1, 3, 2) @ self.cache_placement).permute(0, 1, 3, 2))
            normed = self._rms_norm(hidden, self.weights[f"{w}.post_attention_layernorm.weight"])
            hidden = hidden + self._mlp(normed, layer)
        hidden = self._rms_norm(hidden, self.weights["model.norm.weight"])
        last = (selector @ hidden).reshape(b, c.hidden_size)  # the selector row broadcasts over the prompts
        return (self._linear(last, self.weights["lm_head.weight"]), *caches)


class BatchedRuntime(LlamaRuntime):
    """Prefill B prompts one by one, then decode them together."""

    def __init__(self, config: LlamaConfig, weights, *, batch: int, compiler: str = "cuda-b200",
                 dtype=None) -> None:
        super().__init__(config, weights, compiler=compiler, dtype=dtype)
        self.batch = batch
        self._batched: dict = {}

    def prefill_batch(self, prompts: Sequence[Sequence[int]], context: int, *, temperature: float = 0.0,
                      top_k: int = 50, rng: Optional[np.random.Generator] = None) -> Tuple[List[int], List[Any]]:
        """First token of each prompt (greedy, or sampled with ``rng``) and the stacked (B, ...) caches."""
        if len(prompts) != self.batch or len({len(p) for p in prompts}) != 1:
            raise ValueError(f"{self.batch} prompts of equal length are required")
        logits, caches = self.prefill_batched(prompts, context)  # one program for all prompts
        if temperature == 0:
            return [int(t) for t in self.device.argmax_last_axis(logits)], caches
        rows = logits.tensor.reshape(logits.shape)  # the program's output buffer is flat
        firsts = [self.sample(DeviceArray(rows[i:i + 1], (1,) + tuple(logits.shape[1:]), logits.dtype),
                              temperature, top_k, rng) for i in range(self.batch)]
        return firsts, caches

    def batched_step_inputs(self, tokens: Sequence[int], position: int, context: int) -> List[np.ndarray]:
        c = self.config
        ids = np.asarray(tokens, dtype=np.int32).reshape(-1, 1)
        rotation = _rope_rotations(1, c.head_size, c.rope_theta, self.dtype, offset=position)
        attention, write = decode_masks(position, context, self.dtype)
        return [ids, rotation, attention, write, np.asarray(position, dtype=np.int32)]

    def batched_program(self, context: int, caches: List[Any], tokens: Sequence[int], position: int):
        cached = self._batched.get(context)
        if cached is not None:
            return cached
        host = self.batched_step_inputs(tokens, position, context)
        with no_grad():
            step = BatchedDecoderStep(self.config, self.weights, batch=self.batch, cache_length=context,
                                      dtype=self.dtype)
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

    def decode_batch(self, tokens: Sequence[int], position: int, context: int,
                     caches: List[Any]) -> Tuple[Any, List[Any]]:
        """One step of all sequences: native (B, vocab) logits and the caches."""
        program, nodes = self.batched_program(context, caches, tokens, position)
        values = [self.device.array(v) for v in self.batched_step_inputs(tokens, position, context)]
        produced = program.run(dict(zip(nodes, values + list(caches))), synchronize=False)
        return produced[0], list(produced[1:])

    def generate_batch(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, *,
                       temperature: float = 0.0, top_k: int = 50, seed: int = 0) -> List[List[int]]:
        """Tokens of every sequence (first one from its prefill): greedy at temperature 0, else
        sampled per row on the device, one ``default_rng(seed)`` draw per token in row order."""
        if temperature < 0 or top_k < 0:
            raise ValueError("temperature and top-k cannot be negative")
        rng = np.random.default_rng(seed)
        length = len(prompts[0])
        context = length + max_new_tokens
        tokens, caches = self.prefill_batch(prompts, context, temperature=temperature, top_k=top_k, rng=rng)
        out = [[t] for t in tokens]
        for i in range(1, max_new_tokens):
            logits, caches = self.decode_batch(tokens, length + i - 1, context, caches)
            if temperature == 0:
                tokens = self.greedy_rows(logits)
            else:
                tokens = [int(t) for t in self.device.sample_rows(self.full_logits(logits), temperature=temperature,
                                                                  top_k=top_k, rng=rng)]
            for seq, t in zip(out, tokens):
                seq.append(t)
        return out

    def greedy_rows(self, logits) -> List[int]:
        """The greedy token of every row of ``decode_batch``'s logits (argmax_last_axis)."""
        return [int(t) for t in self.device.argmax_last_axis(logits)]

    def full_logits(self, logits):
        """``decode_batch``'s logits as whole (B, vocab) rows (they already are, here)."""
        return logits

    def _argmax_rows(self, program, logits_view, out_ptr: int, stream: int) -> None:
        """Device argmax of the decode program's logits into ``out_ptr`` (int64 per row), on ``stream``."""
        from . import _lib

        _lib.call("cb_argmax_rows", program.ptr(logits_view), _lib.dtype_code(logits_view.dtype), self.batch,
                  logits_view.shape[-1], out_ptr, stream)

    def decode_batch_on_device(self, tokens: Sequence[int], position: int, context: int, caches: List[Any],
                               steps: int, *, replay_times: Optional[List[float]] = None):
        """Greedy-decode ``steps`` tokens of every sequence with no host round trip per step.

        Two bound runs (the second captures the graph), then ``steps - 1``
        graph replays, each preceded by cb_argmax_rows over the previous
        logits and cb_decode_advance_rows writing the next ids, position and
        masks on the device.  Returns (tokens per sequence, device ms of the
        whole loop); ``replay_times`` receives each replay's device ms.
        """
        import torch

        from . import _lib

        program, nodes = self.batched_program(context, caches, tokens, position)
        self.decode_batch(tokens, position, context, caches)
        self.decode_batch(tokens, position, context, caches)
        ids, _, mask, write, pos = nodes[:5]
        dev = self.device.torch_device
        rows = self.batch
        log = torch.zeros(max(steps, 1) * rows, dtype=torch.int64, device=dev)
        argmax = torch.zeros(rows, dtype=torch.int64, device=dev)
        logits_view = program.plan.outputs[0][1]
        stream = self.device.stream()
        lib = _lib.load()
        slot, code = program.slot_pointer, _lib.dtype_code
        advance = (argmax.data_ptr(), rows, slot(ids), code(ids.dtype), slot(pos), code(pos.dtype), slot(mask),
                   code(program.plan.input_buffers[mask].dtype), slot(write),
                   code(program.plan.input_buffers[write].dtype), context, log.data_ptr())
        marks = ([(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(1, steps)] if replay_times is not None else None)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(1, steps):
            self._argmax_rows(program, logits_view, argmax.data_ptr(), stream)
            _lib.check(lib.cb_decode_advance_rows(*advance, i - 1, program.error_pointer(), stream),
                       "cb_decode_advance_rows")
            if marks is not None:
                marks[i - 1][0].record()
            program.replay(stream)
            if marks is not None:
                marks[i - 1][1].record()
        self._argmax_rows(program, logits_view, log[(steps - 1) * rows:].data_ptr(), stream)
        end.record()
        end.synchronize()
        program.check_errors()
        if marks is not None:
            replay_times.extend(a.elapsed_time(b) for a, b in marks)
        table = log[:steps * rows].view(steps, rows).t().tolist()
        return [[int(t) for t in seq] for seq in table], start.elapsed_time(end)
