"""Parity at the benchmarked shapes, against fixtures made by the reference itself.

* C5 -- the Llama-3-8B shape (head size 128, theta 5e5, vocabulary 128256,
  8 KV heads, intermediate 14336) on two layers: 32-token prompt and 8 greedy
  steps of the reference's ``cpu`` compiler (``llama3_2layer_bf16``), through
  the batch-1 runtime and through the tensor-parallel runtime of the C5
  benchmark at TP = 1 (batched decode, the golden prompt in row 0);
* C4 -- one 2048-token prompt, the prefill workload's length, with
  TinyLlama's per-layer shapes on four layers (``tinyllama_prefill2048``;
  the reference's cpu compiler keeps every intermediate, so all 22 layers do
  not fit a 62 GB host): logits and first token of the reference's prefill,
  through the prefill program (tcgen05 GEMMs, flash attention);
* C3 -- the TinyLlama-shape batch of 32 sequences: the ``tinyllama_bf16``
  golden prompt in row 0 (128 greedy tokens against the reference), every
  other row against its own batch-1 run, logits of one step row by row.

Bars: greedy tokens bit-exact, bf16 logits within 2e-2 absolute.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights
from cuda_b200.runtime import LlamaRuntime

pytestmark = pytest.mark.gpu

BF16_LOGITS = 2e-2


def _bf16_close(got, want):
    err = float(np.max(np.abs(np.asarray(got, np.float32) - np.asarray(want, np.float32))))
    assert err <= BF16_LOGITS, f"max abs logit error {err:.3g}"


@pytest.fixture(scope="module")
def llama3_weights(gpu):
    wl = WORKLOADS["llama3-8b-2layer-bf16"]
    return wl, synthetic_weights(wl.config, dtype=wl.np_dtype)


def test_llama3_shape_prefill_and_greedy_tokens(llama3_weights):
    g = golden("llama3_2layer_bf16")
    wl, weights = llama3_weights
    rt = LlamaRuntime(wl.config, weights, compiler="cuda-b200")
    prompt, context = [int(t) for t in g["prompt"]], int(g["context"])
    logits, caches = rt.prefill(prompt, context)
    _bf16_close(rt.device.to_numpy(logits), g["prefill_logits"])
    tokens = [rt.device.argmax(logits)]
    for i in range(1, len(g["tokens"])):
        logits, caches = rt.decode(tokens[-1], len(prompt) + i - 1, context, caches)
        if f"step{i}_logits" in g:
            _bf16_close(rt.device.to_numpy(logits), g[f"step{i}_logits"])
        tokens.append(rt.device.argmax(logits))
    assert tokens == [int(t) for t in g["tokens"]]


def test_llama3_shape_through_the_tensor_parallel_runtime(llama3_weights):
    """The C5 benchmark's runtime (TensorParallelRuntime, batched decode) at TP = 1."""
    from cuda_b200 import tensor_parallel as tp

    g = golden("llama3_2layer_bf16")
    wl, weights = llama3_weights
    layout = tp.shard_layout(wl.config, 1, 0)
    rt = tp.TensorParallelRuntime(wl.config, tp.shard_weights(wl.config, weights, layout), layout, batch=2)
    prompt = [int(t) for t in g["prompt"]]
    other = [int(t) for t in synthetic_prompt(wl.config, len(prompt), seed=7)[0]]
    steps = len(g["tokens"])
    got = rt.generate_batch([prompt, other], steps)
    assert got[0] == [int(t) for t in g["tokens"]]
    context = int(g["context"])
    tokens, caches = rt.prefill_batch([prompt, other], context)
    logits, _ = rt.decode_batch(tokens, len(prompt), context, caches)
    _bf16_close(rt.device.to_numpy(logits)[0], g["step1_logits"][0])
    rt.close()


def test_tinyllama_prefill_of_2048_tokens(gpu):
    g = golden("tinyllama_prefill2048")
    wl = WORKLOADS["tinyllama-4layer-prefill2048-bf16"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200")
    prompt = [int(t) for t in g["prompt"]]
    assert len(prompt) == 2048
    logits, caches = rt.prefill(prompt, int(g["context"]))
    _bf16_close(rt.device.to_numpy(logits), g["prefill_logits"])
    assert rt.device.argmax(logits) == int(g["tokens"][0])
    fingerprint = np.array([[float(np.sum(np.asarray(c, np.float64))), float(np.sum(np.abs(np.asarray(c, np.float64))))]
                            for c in (rt.device.to_numpy(x) for x in caches)])
    np.testing.assert_allclose(fingerprint[:, 1], g["prefill_cache_fp"][:, 1], rtol=1e-4)
    program = next(iter(rt._prefill.values()))[0]
    assert "matmul_multi" in program.source  # q/k/v, SwiGLU and residual fusions on cb_gemm_tc_multi
    assert all(program._sdpa_tc(s) for s in program.plan.steps if s.name == "sdpa")


def test_tinyllama_batched_prefill_of_2048_token_prompts(gpu):
    """The C4 benchmark's program: four 2048-token prompts as one batched prefill (every Linear
    one GEMM over 8192 rows).  Row 0 is the golden prompt: the reference's logits and first
    token; every row equals its own batch-1 prefill on the GPU (token and logits, caches)."""
    g = golden("tinyllama_prefill2048")
    wl = WORKLOADS["tinyllama-4layer-prefill2048-bf16"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200")
    context = int(g["context"])
    prompts = [[int(t) for t in g["prompt"]]] + [list(p) for p in synthetic_prompt(wl.config, 2048, seed=7, batch=3)]
    logits, caches = rt.prefill_batched(prompts, context)
    rows = rt.device.to_numpy(logits)
    assert rows.shape == (4, wl.config.vocab_size)
    _bf16_close(rows[:1], g["prefill_logits"])
    tokens = [int(t) for t in rt.device.argmax_last_axis(logits)]
    assert tokens[0] == int(g["tokens"][0])
    batched_caches = [rt.device.to_numpy(c) for c in caches]
    for s, prompt in enumerate(prompts):
        one_logits, one_caches = rt.prefill(prompt, context)
        assert rt.device.argmax(one_logits) == tokens[s]
        _bf16_close(rows[s:s + 1], rt.device.to_numpy(one_logits))
        for i, c in enumerate(one_caches):
            want = np.asarray(rt.device.to_numpy(c), np.float32)
            np.testing.assert_allclose(np.asarray(batched_caches[i][s:s + 1], np.float32), want, rtol=0,
                                       atol=1e-3 * max(1.0, float(np.abs(want).max())), err_msg=f"row {s} cache {i}")


def test_tinyllama_batch_of_32(gpu):
    from cuda_b200.batched import BatchedRuntime

    g = golden("tinyllama_bf16")
    wl = WORKLOADS["tinyllama-bf16-bs32"]
    weights = synthetic_weights(wl.config, dtype=wl.np_dtype)
    prompt0 = [int(t) for t in g["prompt"]]
    prompts = [prompt0] + [list(synthetic_prompt(wl.config, len(prompt0), seed=s)[0]) for s in range(1, wl.batch)]
    steps = len(g["tokens"])
    batched = BatchedRuntime(wl.config, weights, batch=wl.batch, compiler="cuda-b200")
    got = batched.generate_batch(prompts, steps)
    assert got[0] == [int(t) for t in g["tokens"]]
    single = LlamaRuntime(wl.config, weights, compiler="cuda-b200")
    for i in range(1, wl.batch):
        assert got[i] == single.generate(prompts[i], steps).tokens, i
    context = len(prompt0) + steps
    tokens, caches = batched.prefill_batch(prompts, context)
    logits, _ = batched.decode_batch(tokens, len(prompt0), context, caches)
    rows = batched.device.to_numpy(logits)
    _bf16_close(rows[0], g["step1_logits"][0])
    for i in range(1, wl.batch, 5):
        one, one_caches = single.prefill(prompts[i], context)
        ref, _ = single.decode(tokens[i], len(prompt0), context, one_caches)
        _bf16_close(rows[i], single.device.to_numpy(ref).reshape(-1))
