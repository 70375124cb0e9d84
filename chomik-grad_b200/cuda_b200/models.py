"""Named model shapes and seeded synthetic weights for the Llama hot path.

There are no checkpoints on the benchmark machines, so every configuration is
random-initialised: non-norm weights ~ N(0, 0.02) drawn in float32 and cast to
the model dtype, RMSNorm weights = 1.  Each tensor has its own generator,
``default_rng(SeedSequence(seed).spawn(n)[k])`` with ``k`` the tensor's index
in ``required_weight_shapes`` order, so tensors are reproducible one by one
and can be drawn on several host threads at once (NumPy releases the GIL while
filling).  Prompts are uniform token ids from ``default_rng(seed + 1)``.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
import os
from typing import Dict, Optional

import numpy as np

from chomikgrad.llama import LlamaConfig, required_weight_shapes


def bfloat16() -> np.dtype:
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


@dataclass(frozen=True)
class Workload:
    """One benchmark/parity configuration of the Llama hot path."""

    name: str
    config: LlamaConfig
    dtype: str              # "float32" | "bfloat16"
    batch: int
    prompt_tokens: int
    decode_steps: int

    @property
    def np_dtype(self) -> np.dtype:
        return np.dtype(np.float32) if self.dtype == "float32" else bfloat16()

    @property
    def context(self) -> int:
        """KV rows per sequence: prompt + generated (generate_tinyllama.py:692)."""
        return self.prompt_tokens + self.decode_steps


TINY = LlamaConfig(vocab_size=4096, hidden_size=256, intermediate_size=688,
                   num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                   max_position_embeddings=128, rope_theta=10_000.0)
TINYLLAMA = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                        num_hidden_layers=22, num_attention_heads=32,
                        num_key_value_heads=4, max_position_embeddings=2048,
                        rope_theta=10_000.0)
LLAMA3_8B = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                        num_hidden_layers=32, num_attention_heads=32,
                        num_key_value_heads=8, max_position_embeddings=8192,
                        rope_theta=500_000.0)
# The Llama-3-8B shape cut to two layers: every per-layer shape, the head size
# 128, theta 5e5 and the 128256-row vocabulary of LLAMA3_8B, at a size the
# reference's cpu compiler runs in minutes (parity fixtures only).
LLAMA3_8B_2L = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                           num_hidden_layers=2, num_attention_heads=32,
                           num_key_value_heads=8, max_position_embeddings=8192,
                           rope_theta=500_000.0)

# The TinyLlama shape cut to four layers: every per-layer shape of TINYLLAMA,
# for the 2048-token prefill fixture (the reference's cpu compiler keeps every
# intermediate of a program alive, about 2.5 GB per layer at 2048 tokens).
TINYLLAMA_4L = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                           num_hidden_layers=4, num_attention_heads=32,
                           num_key_value_heads=4, max_position_embeddings=4096,
                           rope_theta=10_000.0)

WORKLOADS: Dict[str, Workload] = {
    w.name: w
    for w in (
        Workload("tiny-fp32", TINY, "float32", 1, 16, 32),
        Workload("tiny-bf16", TINY, "bfloat16", 1, 16, 32),
        Workload("tinyllama-bf16-bs1", TINYLLAMA, "bfloat16", 1, 128, 256),
        Workload("tinyllama-bf16-bs32", TINYLLAMA, "bfloat16", 32, 512, 256),
        Workload("tinyllama-bf16-prefill-bs8", TINYLLAMA, "bfloat16", 8, 2048, 0),
        Workload("llama3-8b-bf16-bs16", LLAMA3_8B, "bfloat16", 16, 1024, 256),
        Workload("llama3-8b-2layer-bf16", LLAMA3_8B_2L, "bfloat16", 1, 32, 8),
        Workload("tinyllama-4layer-prefill2048-bf16", TINYLLAMA_4L, "bfloat16", 1, 2048, 1),
    )
}


def synthetic_weights(config: LlamaConfig, *, dtype: np.dtype, seed: int = 0,
                      std: float = 0.02, threads: Optional[int] = None) -> Dict[str, np.ndarray]:
    """Seeded random-init weights in HF layout (see module docstring)."""
    dtype = np.dtype(dtype)
    shapes = list(required_weight_shapes(config).items())
    seeds = np.random.SeedSequence(seed).spawn(len(shapes))

    def draw(index: int) -> np.ndarray:
        name, shape = shapes[index]
        if name.endswith("norm.weight"):
            return np.ones(shape, dtype=dtype)
        values = np.random.default_rng(seeds[index]).normal(0.0, std, shape)
        return values.astype(np.float32).astype(dtype)

    workers = threads or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=workers) as pool:
        arrays = list(pool.map(draw, range(len(shapes))))
    return {name: array for (name, _), array in zip(shapes, arrays)}


def synthetic_prompt(config: LlamaConfig, length: int, *, seed: int = 0,
                     batch: int = 1) -> np.ndarray:
    """(batch, length) uniform token ids in [0, vocab)."""
    rng = np.random.default_rng(seed + 1)
    return rng.integers(0, config.vocab_size, size=(batch, length)).astype(np.int32)


def device_weights(config: LlamaConfig, *, device, seed: int = 0, std: float = 0.02, layout=None):
    """Seeded random-init bf16 weights drawn on the GPU (torch), optionally one rank's shards.

    For the large benchmark shapes (Llama-3-8B: 8 billion values), where the
    host-side ``synthetic_weights`` takes minutes.  Tensor k (in
    ``required_weight_shapes`` order) comes from a CUDA generator seeded with
    ``seed * 1000003 + k``; norm weights are 1.  With ``layout`` (a
    ``tensor_parallel.ShardLayout``) each full tensor is drawn, then only this
    rank's shard is kept, so every rank's shards come from the same tensors.
    """
    import torch

    from .tensor_parallel import shard_weights

    out = {}
    gen = torch.Generator(device=device)
    for index, (name, shape) in enumerate(required_weight_shapes(config).items()):
        if name.endswith("norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
            continue
        gen.manual_seed(seed * 1000003 + index)
        full = (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)
        out[name] = shard_weights(config, {name: full}, layout)[name] if layout is not None else full
    return out
