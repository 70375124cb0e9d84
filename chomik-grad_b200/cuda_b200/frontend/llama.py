"""Llama graph builders mirroring ``chomikgrad/llama.py``.

The builders emit the same six-op graphs, with the same preferred lowerings
(``rms_norm`` llama.py:279-287, ``rope`` :293-323, ``sdpa`` :355-364 and
:514-525) and the same constant leaves, as the reference:

* ``LlamaForCausalLM``   -- full causal forward / prefill  (llama.py:212-433)
* ``LlamaDecoderStep``   -- one cached decode step          (llama.py:436-543)
* ``LlamaDecoderBlock``  -- multi-token verify block        (llama.py:546-668)

Graph equality with the reference (node for node, via ``GraphPlan.signature``)
is asserted by the CPU test-suite, which is what makes a program compiled from
these graphs interchangeable with one compiled from the reference's.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Mapping, Optional, Sequence, Tuple

import numpy as np

from .lazy import DeviceAdapter, get_compiler
from .tensor import Tensor

MASKED = -1e4  # additive mask value used by the reference (llama.py:250-258)


def _prefer(output: Tensor, kind: str, inputs: Sequence[Tensor], argument: object) -> Tensor:
    """Attach an optional lowering hint while keeping the portable graph (llama.py:13-25)."""
    output._node.lowering = (kind, tuple(t._node for t in inputs), argument)
    return output


@dataclass(frozen=True)
class LlamaConfig:
    """Architecture hyper-parameters (llama.py:28-97)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10_000.0
    bos_token_id: int = 1
    eos_token_id: int = 2

    _REQUIRED = ("vocab_size", "hidden_size", "intermediate_size",
                 "num_hidden_layers", "num_attention_heads",
                 "num_key_value_heads", "max_position_embeddings")

    @classmethod
    def from_dict(cls, config: Mapping[str, object]) -> "LlamaConfig":
        absent = [key for key in cls._REQUIRED if key not in config]
        if absent:
            raise ValueError(f"missing Llama config fields: {', '.join(absent)}")
        made = cls(**{key: int(config[key]) for key in cls._REQUIRED},
                   rms_norm_eps=float(config.get("rms_norm_eps", 1e-5)),
                   rope_theta=float(config.get("rope_theta", 10_000.0)),
                   bos_token_id=int(config.get("bos_token_id", 1)),
                   eos_token_id=int(config.get("eos_token_id", 2)))
        made.validate()
        return made

    @property
    def head_size(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def query_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def validate(self) -> None:
        if any(getattr(self, key) <= 0 for key in self._REQUIRED):
            raise ValueError("Llama dimensions must be positive")
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden size must be divisible by attention heads")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("attention heads must be divisible by KV heads")
        if self.head_size % 2:
            raise ValueError("RoPE requires an even attention head size")


def required_weight_shapes(config: LlamaConfig) -> Dict[str, Tuple[int, ...]]:
    """HF-style weight names and shapes, in the reference's order (llama.py:100-124)."""
    h, i = config.hidden_size, config.intermediate_size
    kv = config.num_key_value_heads * config.head_size
    shapes: Dict[str, Tuple[int, ...]] = {
        "model.embed_tokens.weight": (config.vocab_size, h),
        "model.norm.weight": (h,),
        "lm_head.weight": (config.vocab_size, h),
    }
    for layer in range(config.num_hidden_layers):
        p = f"model.layers.{layer}"
        shapes[f"{p}.input_layernorm.weight"] = (h,)
        shapes[f"{p}.post_attention_layernorm.weight"] = (h,)
        shapes[f"{p}.self_attn.q_proj.weight"] = (h, h)
        shapes[f"{p}.self_attn.k_proj.weight"] = (kv, h)
        shapes[f"{p}.self_attn.v_proj.weight"] = (kv, h)
        shapes[f"{p}.self_attn.o_proj.weight"] = (h, h)
        shapes[f"{p}.mlp.gate_proj.weight"] = (i, h)
        shapes[f"{p}.mlp.up_proj.weight"] = (i, h)
        shapes[f"{p}.mlp.down_proj.weight"] = (h, i)
    return shapes


def rope_angles(positions: int, head_size: int, theta: float, offset: int = 0) -> np.ndarray:
    """float32 angle table ``pos * theta^(-2j/hd)`` exactly as llama.py:135-140 forms it."""
    where = np.arange(offset, offset + positions, dtype=np.float32)
    inverse = 1.0 / (theta ** (np.arange(0, head_size, 2, dtype=np.float32) / head_size))
    return where[:, None] * inverse[None, :]


def rope_rotations(sequence_length: int, head_size: int, theta: float,
                   dtype: np.dtype, *, offset: int = 0) -> np.ndarray:
    """Dense rotate-half RoPE matrices for row-vector matmul (llama.py:127-152).

    Shape (1, 1, T, hd, hd); column j holds output j's coefficients.
    """
    half = head_size // 2
    angles = rope_angles(sequence_length, head_size, theta, offset)
    cos, sin = np.cos(angles), np.sin(angles)
    table = np.zeros((1, 1, sequence_length, head_size, head_size), dtype=dtype)
    j = np.arange(half)
    table[0, 0, :, j, j] = cos.T
    table[0, 0, :, j + half, j + half] = cos.T
    table[0, 0, :, j, j + half] = sin.T
    table[0, 0, :, j + half, j] = -sin.T
    return table


_rope_rotations = rope_rotations  # reference spelling


def token_one_hot(token_ids: Sequence[int], sequence_length: int, vocab_size: int, *,
                  fill_token_id: int, dtype: np.dtype) -> np.ndarray:
    """(1, T, V) one-hot rows, padded with ``fill_token_id`` (llama.py:155-173)."""
    if len(token_ids) > sequence_length:
        raise ValueError("token sequence exceeds the fixed generation context")
    if not 0 <= fill_token_id < vocab_size:
        raise ValueError("fill token is outside the vocabulary")
    ids = np.full(sequence_length, fill_token_id, dtype=np.int64)
    ids[: len(token_ids)] = token_ids
    if np.any(ids < 0) or np.any(ids >= vocab_size):
        raise ValueError("token id is outside the vocabulary")
    out = np.zeros((1, sequence_length, vocab_size), dtype=dtype)
    out[0, np.arange(sequence_length), ids] = 1
    return out


def position_selector(position: int, sequence_length: int, *, dtype: np.dtype) -> np.ndarray:
    """(1, T) one-hot row selecting the last prompt position (llama.py:176-183)."""
    if not 0 <= position < sequence_length:
        raise ValueError("selected position is outside the generation context")
    out = np.zeros((1, sequence_length), dtype=dtype)
    out[0, position] = 1
    return out


def decode_masks(position: int, context: int, dtype: np.dtype) -> Tuple[np.ndarray, np.ndarray]:
    """Per-step additive attention mask and cache write mask.

    Built the way the generation loop builds them (generate_tinyllama.py:781-786).
    """
    attention = np.full((1, 1, 1, context), MASKED, dtype=dtype)
    attention[..., : position + 1] = 0
    write = np.zeros((1, 1, context, 1), dtype=dtype)
    write[:, :, position, :] = 1
    return attention, write


def load_safetensors(path: Path, device: DeviceAdapter, *,
                     dtype: Optional[np.dtype] = None) -> Dict[str, Tensor]:
    """Wrap a device adapter's safetensors load as native leaves (llama.py:186-203)."""
    loaded = (device.load_safetensors(path) if dtype is None
              else device.load_safetensors(path, dtype=np.dtype(dtype)))
    return {name: Tensor.from_native(value, backend=device.name,
                                     shape=tuple(value.shape),
                                     dtype=device.dtype(value))
            for name, value in loaded.items()}


class LlamaForCausalLM:
    """Llama decoder in six ops: causal forward and cache-collecting prefill."""

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], *,
                 sequence_length: int, dtype: np.dtype,
                 cache_length: Optional[int] = None) -> None:
        config.validate()
        if not 0 < sequence_length <= config.max_position_embeddings:
            raise ValueError("invalid fixed generation context length")
        expected = required_weight_shapes(config)
        for name in expected:
            if name not in weights:
                raise ValueError(f"missing model weight: {name}")
        for name, shape in expected.items():
            if weights[name].shape != shape:
                raise ValueError(
                    f"weight {name} has shape {weights[name].shape}, expected {shape}")
        self.config = config
        self.weights = dict(weights)
        self.sequence_length = sequence_length
        self.dtype = np.dtype(dtype)
        self.cache_length = cache_length
        self.cache_placement: Optional[Tensor] = None
        if cache_length is not None:
            if cache_length < sequence_length:
                raise ValueError("KV cache cannot be shorter than the prompt")
            place = np.zeros((sequence_length, cache_length), dtype=self.dtype)
            place[np.arange(sequence_length), np.arange(sequence_length)] = 1
            self.cache_placement = Tensor(place)
        mask = np.triu(np.full((sequence_length, sequence_length), MASKED, dtype=self.dtype),
                       k=1)
        self.causal_mask = Tensor(mask.reshape(1, 1, sequence_length, sequence_length))
        self.rotations = Tensor(rope_rotations(sequence_length, config.head_size,
                                               config.rope_theta, self.dtype))
        self.kv_repeat = Tensor.ones((1, 1, config.query_groups, 1, 1), dtype=self.dtype)

    @property
    def parameter_count(self) -> int:
        return sum(int(np.prod(w.shape)) for w in self.weights.values())

    # -- building blocks ----------------------------------------------------
    def _w(self, name: str) -> Tensor:
        return self.weights[name]

    @staticmethod
    def _linear(inputs: Tensor, weight: Tensor) -> Tensor:
        """``x @ W.T`` with W in HF (out, in) layout (llama.py:275-277)."""
        return inputs @ weight.T

    def _rms_norm(self, inputs: Tensor, weight: Tensor) -> Tensor:
        """``x / sqrt(mean(x*x) + eps) * w`` + ``rms_norm`` hint (llama.py:279-287)."""
        eps = self.config.rms_norm_eps
        mean_square = (inputs * inputs).mean(axis=-1, keepdims=True)
        scaled = inputs / (mean_square + eps).sqrt() * weight
        return _prefer(scaled, "rms_norm", (inputs, weight), eps)

    @staticmethod
    def _silu(inputs: Tensor) -> Tensor:
        return inputs / (1 + (-inputs).exp())

    def _rotate(self, inputs: Tensor, rotation: Tensor) -> Tensor:
        b, h, t, d = inputs.shape
        return (inputs.reshape(b, h, t, 1, d) @ rotation).reshape(b, h, t, d)

    def _apply_rope(self, inputs: Tensor) -> Tensor:
        """Prefill RoPE against the model's own rotation table (llama.py:293-304)."""
        rotated = self._rotate(inputs, self.rotations)
        return _prefer(rotated, "rope", (inputs,),
                       (inputs.shape[-1], self.config.rope_theta, 0))

    def _apply_rotation(self, inputs: Tensor, rotation: Tensor,
                        position: Optional[Tensor]) -> Tensor:
        """Decode RoPE against a bound rotation; hinted only with a position (llama.py:306-323)."""
        rotated = self._rotate(inputs, rotation)
        if position is None:
            return rotated
        return _prefer(rotated, "rope", (inputs, position),
                       (inputs.shape[-1], self.config.rope_theta, 0))

    def _repeat_kv(self, inputs: Tensor) -> Tensor:
        """GQA broadcast of KV heads to query heads (llama.py:325-330)."""
        b, kv, t, d = inputs.shape
        spread = inputs.reshape(b, kv, 1, t, d) * self.kv_repeat
        return spread.reshape(b, self.config.num_attention_heads, t, d)

    def _attend(self, query: Tensor, keys: Tensor, values: Tensor, mask: Tensor) -> Tensor:
        """Portable masked attention + ``sdpa`` hint over the un-repeated KV."""
        hd = self.config.head_size
        scores = (query @ self._repeat_kv(keys).transpose(-2, -1)) / np.sqrt(hd) + mask
        attended = scores.softmax(axis=-1) @ self._repeat_kv(values)
        return _prefer(attended, "sdpa", (query, keys, values, mask), 1 / np.sqrt(hd))

    def _heads(self, flat: Tensor, tokens: int, heads: int) -> Tensor:
        """(1, T, heads*hd) -> (1, heads, T, hd)."""
        return flat.reshape(1, tokens, heads, self.config.head_size).permute(0, 2, 1, 3)

    def _attention(self, inputs: Tensor, layer: int) -> Tuple[Tensor, Tensor, Tensor]:
        """Prefill self-attention block (llama.py:332-369)."""
        c = self.config
        p = f"model.layers.{layer}.self_attn"
        batch, tokens, _ = inputs.shape
        query = self._linear(inputs, self._w(f"{p}.q_proj.weight"))
        key = self._linear(inputs, self._w(f"{p}.k_proj.weight"))
        value = self._linear(inputs, self._w(f"{p}.v_proj.weight"))
        query = query.reshape(batch, tokens, c.num_attention_heads, c.head_size).permute(0, 2, 1, 3)
        key = key.reshape(batch, tokens, c.num_key_value_heads, c.head_size).permute(0, 2, 1, 3)
        value = value.reshape(batch, tokens, c.num_key_value_heads, c.head_size).permute(0, 2, 1, 3)
        query = self._apply_rope(query)
        key = self._apply_rope(key)
        attended = self._attend(query, key, value, self.causal_mask)
        merged = attended.permute(0, 2, 1, 3).reshape(batch, tokens, c.hidden_size)
        return self._linear(merged, self._w(f"{p}.o_proj.weight")), key, value

    def _mlp(self, inputs: Tensor, layer: int) -> Tensor:
        """SwiGLU feed-forward (llama.py:371-380)."""
        p = f"model.layers.{layer}.mlp"
        gate = self._silu(self._linear(inputs, self._w(f"{p}.gate_proj.weight")))
        up = self._linear(inputs, self._w(f"{p}.up_proj.weight"))
        return self._linear(gate * up, self._w(f"{p}.down_proj.weight"))

    def _embed(self, token_matrix: Tensor) -> Tensor:
        table = self._w("model.embed_tokens.weight")
        if token_matrix.ndim == 2:
            return table.gather(token_matrix)
        return token_matrix @ table

    def _place(self, rows: Tensor, placement: Tensor) -> Tensor:
        """Scatter (1, kv, T, hd) rows into cache positions by ``placement`` matmul."""
        return (rows.permute(0, 1, 3, 2) @ placement).permute(0, 1, 3, 2)

    def _forward(self, token_matrix: Tensor, selector: Tensor, *,
                 collect_cache: bool) -> Tuple[Tensor, ...]:
        """Causal forward over the fixed context (llama.py:382-427)."""
        s, c = self.sequence_length, self.config
        if token_matrix.shape not in ((1, s), (1, s, c.vocab_size)):
            raise ValueError("token matrix has the wrong fixed-context shape")
        if selector.shape != (1, s):
            raise ValueError("position selector has the wrong shape")
        hidden = self._embed(token_matrix)
        caches = []
        for layer in range(c.num_hidden_layers):
            p = f"model.layers.{layer}"
            normed = self._rms_norm(hidden, self._w(f"{p}.input_layernorm.weight"))
            attended, key, value = self._attention(normed, layer)
            hidden = hidden + attended
            if collect_cache:
                if self.cache_placement is None:
                    raise RuntimeError("prefill requires a configured KV cache length")
                caches.append(self._place(key, self.cache_placement))
                caches.append(self._place(value, self.cache_placement))
            normed = self._rms_norm(hidden, self._w(f"{p}.post_attention_layernorm.weight"))
            hidden = hidden + self._mlp(normed, layer)
        hidden = self._rms_norm(hidden, self._w("model.norm.weight"))
        picked = (selector @ hidden).reshape(1, c.hidden_size)
        return (self._linear(picked, self._w("lm_head.weight")), *caches)

    def __call__(self, token_matrix: Tensor, selector: Tensor) -> Tensor:
        return self._forward(token_matrix, selector, collect_cache=False)[0]

    def prefill(self, token_matrix: Tensor, selector: Tensor) -> Tuple[Tensor, ...]:
        """Logits of the selected position plus 2L KV caches of ``cache_length`` rows."""
        return self._forward(token_matrix, selector, collect_cache=True)


class LlamaDecoderStep(LlamaForCausalLM):
    """One cached decode step (llama.py:436-543)."""

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], *,
                 cache_length: int, dtype: np.dtype) -> None:
        super().__init__(config, weights, sequence_length=1, dtype=dtype)
        if not 0 < cache_length <= config.max_position_embeddings:
            raise ValueError("invalid KV cache length")
        self.cache_length = cache_length

    def __call__(self, token_matrix: Tensor, rotation: Tensor, attention_mask: Tensor,
                 write_mask: Tensor, caches: Sequence[Tuple[Tensor, Tensor]], *,
                 position: Optional[Tensor] = None) -> Tuple[Tensor, ...]:
        c, ctx = self.config, self.cache_length
        if token_matrix.shape not in ((1, 1), (1, 1, c.vocab_size)):
            raise ValueError("decode token matrix must contain exactly one token")
        if rotation.shape != (1, 1, 1, c.head_size, c.head_size):
            raise ValueError("decode RoPE rotation has the wrong shape")
        if attention_mask.shape != (1, 1, 1, ctx):
            raise ValueError("decode attention mask has the wrong shape")
        if write_mask.shape != (1, 1, ctx, 1):
            raise ValueError("decode cache write mask has the wrong shape")
        if len(caches) != c.num_hidden_layers:
            raise ValueError("decode requires one KV cache pair per layer")
        if position is not None and position.shape != ():
            raise ValueError("decode position must be a scalar")

        hidden = self._embed(token_matrix)
        updated = []
        cache_shape = (1, c.num_key_value_heads, ctx, c.head_size)
        for layer, (old_key, old_value) in enumerate(caches):
            if old_key.shape != cache_shape or old_value.shape != cache_shape:
                raise ValueError("KV cache has the wrong shape")
            p = f"model.layers.{layer}"
            a = f"{p}.self_attn"
            normed = self._rms_norm(hidden, self._w(f"{p}.input_layernorm.weight"))
            query = self._linear(normed, self._w(f"{a}.q_proj.weight")).reshape(
                1, c.num_attention_heads, 1, c.head_size)
            key = self._linear(normed, self._w(f"{a}.k_proj.weight")).reshape(
                1, c.num_key_value_heads, 1, c.head_size)
            value = self._linear(normed, self._w(f"{a}.v_proj.weight")).reshape(
                1, c.num_key_value_heads, 1, c.head_size)
            query = self._apply_rotation(query, rotation, position)
            key = self._apply_rotation(key, rotation, position)
            new_key = old_key * (1 - write_mask) + key * write_mask
            new_value = old_value * (1 - write_mask) + value * write_mask
            updated.extend((new_key, new_value))
            attended = self._attend(query, new_key, new_value, attention_mask)
            merged = attended.permute(0, 2, 1, 3).reshape(1, 1, c.hidden_size)
            hidden = hidden + self._linear(merged, self._w(f"{a}.o_proj.weight"))
            normed = self._rms_norm(hidden, self._w(f"{p}.post_attention_layernorm.weight"))
            hidden = hidden + self._mlp(normed, layer)

        hidden = self._rms_norm(hidden, self._w("model.norm.weight"))
        logits = self._linear(hidden.reshape(1, c.hidden_size), self._w("lm_head.weight"))
        return (logits, *updated)


class LlamaDecoderBlock(LlamaForCausalLM):
    """Verify ``block_length`` cached positions in one graph (llama.py:546-668)."""

    def __init__(self, config: LlamaConfig, weights: Mapping[str, Tensor], *,
                 block_length: int, cache_length: int, dtype: np.dtype) -> None:
        super().__init__(config, weights, sequence_length=block_length, dtype=dtype)
        if cache_length < block_length or cache_length > config.max_position_embeddings:
            raise ValueError("invalid KV cache length")
        self.block_length = block_length
        self.cache_length = cache_length

    def __call__(self, token_matrix: Tensor, rotation: Tensor, attention_mask: Tensor,
                 cache_placement: Tensor, write_mask: Tensor,
                 caches: Sequence[Tuple[Tensor, Tensor]], *,
                 position: Optional[Tensor] = None) -> Tuple[Tensor, ...]:
        c, ctx, t = self.config, self.cache_length, self.block_length
        if token_matrix.shape not in ((1, t), (1, t, c.vocab_size)):
            raise ValueError("decode block has the wrong token shape")
        if rotation.shape != (1, 1, t, c.head_size, c.head_size):
            raise ValueError("decode block RoPE rotation has the wrong shape")
        if attention_mask.shape != (1, 1, t, ctx):
            raise ValueError("decode block attention mask has the wrong shape")
        if cache_placement.shape != (t, ctx):
            raise ValueError("decode block cache placement has the wrong shape")
        if write_mask.shape != (1, 1, ctx, 1):
            raise ValueError("decode block write mask has the wrong shape")
        if len(caches) != c.num_hidden_layers:
            raise ValueError("decode block requires one KV cache pair per layer")
        if position is not None and position.shape != ():
            raise ValueError("decode block position must be a scalar")

        hidden = self._embed(token_matrix)
        updated = []
        cache_shape = (1, c.num_key_value_heads, ctx, c.head_size)
        for layer, (old_key, old_value) in enumerate(caches):
            if old_key.shape != cache_shape or old_value.shape != cache_shape:
                raise ValueError("KV cache has the wrong shape")
            p = f"model.layers.{layer}"
            a = f"{p}.self_attn"
            normed = self._rms_norm(hidden, self._w(f"{p}.input_layernorm.weight"))
            query = self._linear(normed, self._w(f"{a}.q_proj.weight")).reshape(
                1, t, c.num_attention_heads, c.head_size).permute(0, 2, 1, 3)
            key = self._linear(normed, self._w(f"{a}.k_proj.weight")).reshape(
                1, t, c.num_key_value_heads, c.head_size).permute(0, 2, 1, 3)
            value = self._linear(normed, self._w(f"{a}.v_proj.weight")).reshape(
                1, t, c.num_key_value_heads, c.head_size).permute(0, 2, 1, 3)
            query = self._apply_rotation(query, rotation, position)
            key = self._apply_rotation(key, rotation, position)
            new_key = old_key * (1 - write_mask) + self._place(key, cache_placement)
            new_value = old_value * (1 - write_mask) + self._place(value, cache_placement)
            updated.extend((new_key, new_value))
            attended = self._attend(query, new_key, new_value, attention_mask)
            merged = attended.permute(0, 2, 1, 3).reshape(1, t, c.hidden_size)
            hidden = hidden + self._linear(merged, self._w(f"{a}.o_proj.weight"))
            normed = self._rms_norm(hidden, self._w(f"{p}.post_attention_layernorm.weight"))
            hidden = hidden + self._mlp(normed, layer)

        hidden = self._rms_norm(hidden, self._w("model.norm.weight"))
        logits = self._linear(hidden, self._w("lm_head.weight"))
        return (logits, *updated)
