"""Batched greedy decode (cuda_b200.batched) against batch-1 decode of each sequence.

Per sequence the batched step is the reference's LlamaDecoderStep
(chomikgrad/llama.py:436-543); only the weight reads are shared.  Bars: the
greedy tokens of every sequence equal its batch-1 run (which the golden
tests pin to the reference), logits within the plugin's bars (float32:
max relative 1e-4; bfloat16 model: 2e-2 absolute).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights
from cuda_b200.runtime import LlamaRuntime

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,batch", [("tiny-bf16", 4), ("tiny-fp32", 3), ("tiny-bf16", 32)])
def test_batched_decode_matches_batch_one(gpu, name, batch):
    from cuda_b200.batched import BatchedRuntime

    wl = WORKLOADS[name]
    weights = synthetic_weights(wl.config, dtype=wl.np_dtype)
    g = golden(name.replace("-", "_"))
    prompt0 = [int(t) for t in g["prompt"]]
    prompts = [prompt0] + [list(synthetic_prompt(wl.config, len(prompt0), seed=s)[0]) for s in range(1, batch)]
    steps = len(g["tokens"])  # the golden's context, so the split layout of the attention matches
    batched = BatchedRuntime(wl.config, weights, batch=batch, compiler="cuda-b200")
    single = LlamaRuntime(wl.config, weights, compiler="cuda-b200")
    got = batched.generate_batch(prompts, steps)
    for i, prompt in enumerate(prompts):
        assert got[i] == single.generate(prompt, steps).tokens, i
    assert got[0] == [int(t) for t in g["tokens"]]
    # logits of one step, every row against its own batch-1 step
    context = len(prompt0) + steps
    tokens, caches = batched.prefill_batch(prompts, context)
    logits, _ = batched.decode_batch(tokens, len(prompt0), context, caches)
    rows = batched.device.to_numpy(logits)
    for i, prompt in enumerate(prompts):
        one, one_caches = single.prefill(prompt, context)
        ref, _ = single.decode(tokens[i], len(prompt0), context, one_caches)
        ref = single.device.to_numpy(ref).reshape(-1)
        if wl.np_dtype == np.float32:
            assert np.max(np.abs(rows[i] - ref)) / np.max(np.abs(ref)) <= 1e-4
        else:
            assert np.max(np.abs(rows[i] - ref)) <= 2e-2
    program = next(iter(batched._batched.values()))[0]
    # the caches are blended in place (by the fused batched attention when the q/k/v projections
    # run on the bf16 row GEMM, else by cb_kv_write) and returned aliased
    fused = "decode_attention_batched" in program.source
    assert fused == (wl.np_dtype != np.float32)
    assert (fused or "kv_write" in program.source) and program.plan.aliases


def test_batched_on_device_loop_matches_host_loop(gpu):
    """Graph replays driven by cb_argmax_rows + cb_decode_advance_rows give the host loop's tokens."""
    from cuda_b200.batched import BatchedRuntime

    wl = WORKLOADS["tiny-bf16"]
    weights = synthetic_weights(wl.config, dtype=wl.np_dtype)
    batch, length, steps = 5, 16, 20
    prompts = [list(synthetic_prompt(wl.config, length, seed=40 + s)[0]) for s in range(batch)]
    rt = BatchedRuntime(wl.config, weights, batch=batch, compiler="cuda-b200")
    want = rt.generate_batch(prompts, steps)
    context = length + steps
    tokens, caches = rt.prefill_batch(prompts, context)
    got, ms = rt.decode_batch_on_device(tokens, length, context, caches, steps - 1)
    assert ms > 0
    for i in range(batch):
        assert [tokens[i]] + got[i] == want[i][:steps], i
