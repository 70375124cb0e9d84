"""Greedy Llama generation through the public plugin contract.

``LlamaRuntime`` is the caller side of the hot path, restating the loop of
``examples/generate_tinyllama.py`` (``TinyLlamaRuntime`` :165-263 and
``_generate_loaded`` :678-857) without tokenizer or checkpoint download:

* the prefill graph is compiled once per (prompt length, context) with the
  token ids as the dynamic input (:727-750);
* the decode step graph is compiled once per context with tokens, rotation,
  attention mask, write mask, position and the 2L caches as dynamic inputs
  (:788-842) and replayed with fresh host inputs every step;
* the token is ``device.argmax`` of the step's logits at temperature 0, else
  the device's temperature / top-k sampler with the reference's seeded
  generator (:124-157, :712);
* the caches returned by step n are bound as inputs of step n+1 (:857).

The graphs are the reference package's own (``chomikgrad.llama``
``LlamaForCausalLM.prefill`` and ``LlamaDecoderStep``), compiled through
``chomikgrad.compile_graph``.  It works with any compiler registered in
``chomikgrad``'s registry: ``cuda-b200`` for the product path, the parity
oracle or the reference's own ``cpu`` compiler in tests.
"""

from __future__ import annotations

from dataclasses import dataclass, field
import time
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from chomikgrad.lazy import get_compiler
from chomikgrad.llama import LlamaConfig, LlamaDecoderStep, LlamaForCausalLM, _rope_rotations, position_selector
from chomikgrad.tensor import Tensor, compile_graph, no_grad

from .graphs import decode_masks


@dataclass
class GenerationResult:
    tokens: List[int]
    first_token_seconds: float
    step_seconds: List[float] = field(default_factory=list)

    @property
    def warm_tokens_per_second(self) -> Optional[float]:
        warm = self.step_seconds
        return len(warm) / sum(warm) if warm else None


class LlamaRuntime:
    """Model state reused across generation requests (generate_tinyllama.py:165-263)."""

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Any], *,
                 compiler: str = "cuda-b200", dtype: Optional[np.dtype] = None) -> None:
        self.config = config
        self.compiler_name = compiler
        self.device = get_compiler(compiler).device
        first = next(iter(weights.values()))
        self.dtype = np.dtype(dtype if dtype is not None else
                              (first.dtype if isinstance(first, Tensor) else np.asarray(first).dtype))
        self.weights: Dict[str, Tensor] = {}
        for name, value in weights.items():
            if isinstance(value, Tensor):
                self.weights[name] = value
            else:
                native = self.device.array(value)
                self.weights[name] = Tensor.from_native(
                    native, backend=self.device.name, shape=tuple(native.shape),
                    dtype=self.device.dtype(native))
        self._prefill: Dict[Tuple[int, int], Tuple[Any, Any]] = {}
        self._decoders: Dict[int, Tuple[Any, List[Any]]] = {}
        self._ahead: Optional[Tuple[Tuple[int, int], List[Any]]] = None

    # -- one program each -------------------------------------------------
    def prefill(self, prompt_ids: Sequence[int], context: int) -> Tuple[Any, List[Any]]:
        """Run the prompt; returns native logits and 2L native caches."""
        ids = np.asarray(prompt_ids, dtype=np.int32).reshape(1, -1)
        key = (ids.shape[1], context)
        cached = self._prefill.get(key)
        with no_grad():
            if cached is None:
                model = LlamaForCausalLM(self.config, self.weights,
                                         sequence_length=ids.shape[1], dtype=self.dtype,
                                         cache_length=context)
                selector = position_selector(ids.shape[1] - 1, ids.shape[1], dtype=self.dtype)
                source = Tensor(ids, copy=False)
                outputs = model.prefill(source, Tensor(selector, copy=False))
                program = compile_graph(*outputs, compiler=self.compiler_name,
                                        dynamic_inputs=(source,))
                self._prefill[key] = (program, source._node)
                bindings = None
            else:
                program, node = cached
                bindings = {node: self.device.array(ids)}
            produced = program.run(bindings, synchronize=False)
        return produced[0], list(produced[1:])

    def prefill_batched(self, prompts: Sequence[Sequence[int]], context: int) -> Tuple[Any, List[Any]]:
        """B prompts of equal length as one program (``batched.BatchedPrefill``): native
        (B, vocab) logits of each prompt's last token and 2L native (B, kv_heads, context,
        head_size) caches.  Per prompt the same values as ``prefill``; every Linear runs as one
        GEMM over all B * T rows."""
        from .batched import BatchedPrefill

        ids = np.asarray(prompts, dtype=np.int32)
        if ids.ndim != 2 or ids.shape[0] == 0:
            raise ValueError("prompts must be a non-empty list of equal-length token lists")
        key = ("batched",) + ids.shape + (context,)
        cached = self._prefill.get(key)
        with no_grad():
            if cached is None:
                b, t = ids.shape
                model = BatchedPrefill(self.config, self.weights, batch=b, sequence_length=t, dtype=self.dtype,
                                       cache_length=context)
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

    def step_inputs(self, token: int, position: int, context: int) -> List[np.ndarray]:
        """Host inputs of one decode step, built as generate_tinyllama.py:773-786 builds them."""
        return [np.asarray([[token]], dtype=np.int32), *self._position_host(position, context)]

    def _position_host(self, position: int, context: int) -> List[np.ndarray]:
        """The inputs of a step that depend on its position only: rotation, masks, position."""
        c = self.config
        rotation = _rope_rotations(1, c.head_size, c.rope_theta, self.dtype, offset=position)
        attention, write = decode_masks(position, context, self.dtype)
        return [rotation, attention, write, np.asarray(position, dtype=np.int32)]

    def _position_values(self, position: int, context: int) -> List[Any]:
        """Native position inputs of a step: prepared by the previous decode() while the device ran it."""
        ahead = self._ahead
        self._ahead = None
        if ahead is not None and ahead[0] == (position, context):
            return ahead[1]
        return [self.device.array(v) for v in self._position_host(position, context)]

    def decode_program(self, context: int, caches: List[Any], token: int, position: int):
        """The cached decode program for ``context`` (compiled on first use)."""
        cached = self._decoders.get(context)
        if cached is not None:
            return cached
        c = self.config
        host = self.step_inputs(token, position, context)
        with no_grad():
            step = LlamaDecoderStep(c, self.weights, cache_length=context, dtype=self.dtype)
            tensors = [Tensor(v, copy=False) for v in host]
            cache_tensors = [Tensor.from_native(v, backend=self.device.name,
                                                shape=tuple(v.shape), dtype=self.dtype)
                             for v in caches]
            outputs = step(tensors[0], tensors[1], tensors[2], tensors[3],
                           list(zip(cache_tensors[::2], cache_tensors[1::2])),
                           position=tensors[4])
            dynamic = [*tensors, *cache_tensors]
            program = compile_graph(*outputs, compiler=self.compiler_name,
                                    dynamic_inputs=dynamic)
        entry = (program, [t._node for t in dynamic])
        self._decoders[context] = entry
        return entry

    def decode(self, token: int, position: int, context: int,
               caches: List[Any]) -> Tuple[Any, List[Any]]:
        """One cached step: bind fresh host inputs and the previous caches.

        The next position's rotation and masks (they do not depend on the
        token) are built after the launch, while the device runs this step,
        so the host's share of the step is shorter; the token id is bound
        when it is known.
        """
        program, nodes = self.decode_program(context, caches, token, position)
        values = [self.device.array(np.asarray([[token]], dtype=np.int32)),
                  *self._position_values(position, context)]
        produced = program.run(dict(zip(nodes, values + list(caches))), synchronize=False)
        if position + 1 < context:
            nxt = position + 1
            self._ahead = ((nxt, context), [self.device.array(v) for v in self._position_host(nxt, context)])
        return produced[0], list(produced[1:])

    def decode_on_device(self, token: int, position: int, context: int, caches: List[Any],
                         steps: int, *, timed: bool = False, replay_times: Optional[List[float]] = None):
        """Greedy-decode ``steps`` tokens with no host round trip per token.

        The decode program runs once normally (binding ``token``/``position``
        and the caches), then ``steps - 1`` more times as graph replays with
        ``cb_decode_advance`` writing each next step's inputs from the
        previous argmax.  Only for the ``cuda-b200`` compiler.  Returns the
        tokens (and, with ``timed``, the device milliseconds of the replays).
        With ``replay_times``, CUDA events around every replay append each
        replay's device milliseconds (the decode-step kernel alone when the
        program runs as one cb_decode_step launch).
        """
        import torch

        from . import _lib

        program, nodes = self.decode_program(context, caches, token, position)
        # two bound runs: the second one captures the graph that replay() reuses
        logits, caches = self.decode(token, position, context, caches)
        logits, caches = self.decode(token, position, context, caches)
        ids, _, mask, write, pos = nodes[:5]
        dev = self.device.torch_device
        log = torch.zeros(max(steps, 1), dtype=torch.int64, device=dev)
        stream = self.device.stream()
        lib = _lib.load()
        argmax = program.argmax_pointer(0)
        slot = program.slot_pointer
        code = _lib.dtype_code
        args = (argmax, slot(ids), code(ids.dtype), slot(pos), code(pos.dtype), slot(mask),
                code(program.plan.input_buffers[mask].dtype), slot(write),
                code(program.plan.input_buffers[write].dtype), context, log.data_ptr())
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        marks = ([(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(1, steps)] if replay_times is not None else None)
        start.record()
        # advance i logs the token of the step that just ran (position + i - 1)
        for i in range(1, steps):
            _lib.check(lib.cb_decode_advance(*args, i - 1, program.error_pointer(), stream),
                       "cb_decode_advance")
            if marks is not None:
                marks[i - 1][0].record()
            program.replay(stream)
            if marks is not None:
                marks[i - 1][1].record()
        end.record()
        final = program._tensors[program.plan.argmax_of[0]]
        log[steps - 1:steps].copy_(final[:1])
        end.synchronize()
        program.check_errors()
        if marks is not None:
            replay_times.extend(a.elapsed_time(b) for a, b in marks)
        tokens = [int(t) for t in log[:steps].tolist()]
        return (tokens, start.elapsed_time(end)) if timed else tokens

    # -- the loop ---------------------------------------------------------
    def sample(self, logits: Any, temperature: float, top_k: int, rng: np.random.Generator) -> int:
        """sample_native_token (generate_tinyllama.py:146-157): argmax at temperature 0, else the
        device's sampler (cb_sample_rows on cuda-b200: one draw up, one token down)."""
        if temperature == 0:
            return self.device.argmax(logits)
        return int(self.device.sample(logits, temperature=temperature, top_k=top_k, rng=rng))

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int, *,
                 stop_at_eos: bool = False, temperature: float = 0.0, top_k: int = 50,
                 seed: int = 0) -> GenerationResult:
        """Decode like generate_tinyllama.py:678-857 (greedy at temperature 0, the default).

        The sampler's generator is ``np.random.default_rng(seed)`` (:712),
        drawn once per sampled token, so a run consumes the same random
        stream as the reference's with the same seed.
        """
        if temperature < 0:
            raise ValueError("temperature cannot be negative")
        if top_k < 0:
            raise ValueError("top-k cannot be negative")
        rng = np.random.default_rng(seed)
        prompt = [int(t) for t in prompt_ids]
        if not prompt:
            raise ValueError("the prompt produced no tokens")
        context = len(prompt) + max_new_tokens
        if context > self.config.max_position_embeddings:
            raise ValueError(f"prompt plus output is {context} tokens, model limit is "
                             f"{self.config.max_position_embeddings}")
        started = time.perf_counter()
        logits, caches = self.prefill(prompt, context)
        token = self.sample(logits, temperature, top_k, rng)
        result = GenerationResult([token], time.perf_counter() - started)
        tokens = prompt + [token]
        for _ in range(1, max_new_tokens):
            if stop_at_eos and token == self.config.eos_token_id:
                break
            begun = time.perf_counter()
            logits, caches = self.decode(token, len(tokens) - 1, context, caches)
            token = self.sample(logits, temperature, top_k, rng)
            result.step_seconds.append(time.perf_counter() - begun)
            tokens.append(token)
            result.tokens.append(token)
        return result
