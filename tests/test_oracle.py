"""The parity oracle is pinned to the reference: it must reproduce the golden
fixtures (made by the reference's own cpu compiler) bit for bit."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from chomikgrad.tensor import Tensor
from cuda_b200.models import WORKLOADS, synthetic_weights
from cuda_b200.runtime import LlamaRuntime


def bf16():
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


def test_six_op_known_answers(oracle):
    g = golden("six_ops")
    r = (((Tensor(g["chain_left"]) @ Tensor(g["chain_right"])).relu() + 0.25)
         .permute(1, 0).reshape(1, 4).sum(axis=1))
    assert np.array_equal(r.numpy(compiler="cpu"), g["chain_out"])
    gathered = Tensor(g["gather_table"]).gather(Tensor(g["gather_idx"], copy=False))
    assert np.array_equal(gathered.numpy(compiler="cpu"), g["gather_out"])
    assert np.array_equal((Tensor(g["bmm_a"]) @ Tensor(g["bmm_b"])).numpy(compiler="cpu"), g["bmm_out"])
    assert np.array_equal(Tensor(g["softmax_x"]).softmax(axis=-1).numpy(compiler="cpu"), g["softmax_out"])
    x = g["bf16_sumsq_x"].view(bf16())
    t = Tensor(x)
    out = (t * t).sum(axis=-1, keepdims=True).numpy(compiler="cpu")
    assert np.array_equal(out.view(np.uint16), g["bf16_sumsq_out"])


def test_bf16_sum_is_sequential_in_the_reference_semantics(oracle):
    """ml_dtypes reduces bfloat16 in index order with per-add rounding (the
    stagnation the fused norm kernels reproduce)."""
    x = np.random.default_rng(0).normal(0, 0.02, 2048).astype(np.float32).astype(bf16())
    t = Tensor(x)
    got = (t * t).sum().numpy(compiler="cpu")
    sq = x * x
    acc = sq[0]
    for v in sq[1:]:
        acc = (np.float32(acc) + np.float32(v)).astype(bf16())
    assert got == acc
    assert float(got) < 0.8 * float(np.sum(sq.astype(np.float32)))


@pytest.mark.parametrize("name", ["tiny_fp32", "tiny_bf16"])
def test_oracle_generation_is_bit_identical_to_reference(oracle, name):
    g = golden(name)
    wl = WORKLOADS[name.replace("_", "-")]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cpu")
    context = int(g["context"])
    logits, caches = rt.prefill(list(g["prompt"]), context)
    assert np.array_equal(np.asarray(logits, np.float32), g["prefill_logits"])
    result = rt.generate(list(g["prompt"]), len(g["tokens"]))
    assert result.tokens == [int(t) for t in g["tokens"]]


def test_oracle_tinyllama_prefill_logits(oracle):
    """Full-size bf16 prefill (22 layers, 128 tokens) through the oracle."""
    g = golden("tinyllama_bf16")
    wl = WORKLOADS["tinyllama-bf16-bs1"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cpu")
    logits, _ = rt.prefill(list(g["prompt"]), int(g["context"]))
    assert np.array_equal(np.asarray(logits, np.float32), g["prefill_logits"])
    assert int(np.argmax(logits)) == int(g["tokens"][0])
