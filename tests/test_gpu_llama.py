"""End-to-end Llama parity on the GPU against the reference's golden outputs.

Bars (from the plugin's specification):
  * greedy token ids: bit-exact;
  * float32 logits: max relative error <= 1e-4 (max|a-b| / max|b|);
  * bfloat16 logits: within 2e-2 absolute;
The runtime drives prefill + decode exactly like
examples/generate_tinyllama.py:_generate_loaded (temperature 0, no EOS stop).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from chomikgrad.tensor import Tensor, compile_graph
from cuda_b200.models import WORKLOADS, synthetic_weights
from cuda_b200.runtime import LlamaRuntime

pytestmark = pytest.mark.gpu


def max_rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


def _runtime(name):
    wl = WORKLOADS[name]
    return LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200")


@pytest.fixture(scope="module")
def tiny_fp32(gpu):
    return _runtime("tiny-fp32")


def test_tiny_fp32_generation_matches_reference(tiny_fp32):
    g = golden("tiny_fp32")
    rt = tiny_fp32
    steps = len(g["tokens"])
    context = int(g["context"])
    logits, caches = rt.prefill(list(g["prompt"]), context)
    assert max_rel(rt.device.to_numpy(logits), g["prefill_logits"]) <= 1e-4
    tokens = [rt.device.argmax(logits)]
    prompt = list(g["prompt"])
    for i in range(1, steps):
        logits, caches = rt.decode(tokens[-1], len(prompt) + i - 1, context, caches)
        if f"step{i}_logits" in g:
            assert max_rel(rt.device.to_numpy(logits), g[f"step{i}_logits"]) <= 1e-4
        tokens.append(rt.device.argmax(logits))
    assert tokens == [int(t) for t in g["tokens"]]


def test_tiny_fp32_decode_program_is_fused(tiny_fp32):
    program, _ = next(iter(tiny_fp32._decoders.values()))
    src = program.source
    for name in ("gemv_store", "decode_attention", "gemv_residual", "gemv_silu_mul", "gemv_argmax"):
        assert name in src, name
    assert "matmul(" not in src and "elementwise(" not in src
    assert program.plan.aliases, "KV caches should be updated in place"


def test_tiny_bf16_generation_matches_reference(gpu):
    g = golden("tiny_bf16")
    rt = _runtime("tiny-bf16")
    result = rt.generate(list(g["prompt"]), len(g["tokens"]))
    assert result.tokens == [int(t) for t in g["tokens"]]
    logits, _ = rt.prefill(list(g["prompt"]), int(g["context"]))
    assert np.max(np.abs(rt.device.to_numpy(logits) - g["prefill_logits"])) <= 2e-2


def test_on_device_decode_loop_matches_host_loop(tiny_fp32):
    g = golden("tiny_fp32")
    rt = tiny_fp32
    prompt = list(g["prompt"])
    context = int(g["context"])
    logits, caches = rt.prefill(prompt, context)
    first = rt.device.argmax(logits)
    tokens = rt.decode_on_device(first, len(prompt), context, caches, len(g["tokens"]) - 1)
    assert [first] + tokens == [int(t) for t in g["tokens"]]


def test_returned_caches_are_the_bound_buffers(tiny_fp32):
    rt = tiny_fp32
    g = golden("tiny_fp32")
    logits, caches = rt.prefill(list(g["prompt"]), int(g["context"]))
    token = rt.device.argmax(logits)
    _, updated = rt.decode(token, len(g["prompt"]), int(g["context"]), caches)
    assert all(a is b for a, b in zip(updated, caches))


def test_block_decode_matches_reference(gpu, oracle):
    from chomikgrad import llama as L

    g = golden("tiny_block")
    wl = WORKLOADS["tiny-fp32"]
    cfg = wl.config
    weights = {n: Tensor(v) for n, v in synthetic_weights(cfg, dtype=np.float32).items()}
    prompt, proposed = list(g["prompt"]), list(g["proposed"])
    ctx = len(prompt) + len(proposed)
    pre = L.LlamaForCausalLM(cfg, weights, sequence_length=len(prompt), cache_length=ctx, dtype=np.float32)
    native = compile_graph(*pre.prefill(Tensor(np.asarray([prompt], dtype=np.int32), copy=False),
                                        Tensor(L.position_selector(len(prompt) - 1, len(prompt),
                                                                   dtype=np.float32))),
                           compiler="cuda-b200")()
    caches = [(Tensor(native[i]), Tensor(native[i + 1])) for i in range(1, len(native), 2)]
    t, start = len(proposed), len(prompt)
    placement = np.zeros((t, ctx), dtype=np.float32)
    placement[np.arange(t), start + np.arange(t)] = 1
    write = placement.sum(axis=0).reshape(1, 1, ctx, 1)
    mask = np.full((1, 1, t, ctx), -1e4, dtype=np.float32)
    for i in range(t):
        mask[0, 0, i, : start + i + 1] = 0
    block = L.LlamaDecoderBlock(cfg, weights, block_length=t, cache_length=ctx, dtype=np.float32)
    got = compile_graph(*block(Tensor(np.asarray([proposed], dtype=np.int32), copy=False),
                               Tensor(L._rope_rotations(t, cfg.head_size, cfg.rope_theta,
                                                       np.dtype(np.float32), offset=start)),
                               Tensor(mask), Tensor(placement), Tensor(write), caches),
                        compiler="cuda-b200")()
    assert max_rel(got[0], g["logits"]) <= 1e-4
    np.testing.assert_allclose(got[1], g["cache0"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(got[-1], g["cache_last"], rtol=1e-4, atol=1e-6)


def test_tinyllama_bf16_prefill_and_128_greedy_tokens(gpu):
    g = golden("tinyllama_bf16")
    rt = _runtime("tinyllama-bf16-bs1")
    prompt = list(g["prompt"])
    context = int(g["context"])
    logits, caches = rt.prefill(prompt, context)
    assert np.max(np.abs(rt.device.to_numpy(logits) - g["prefill_logits"])) <= 2e-2
    result = rt.generate(prompt, len(g["tokens"]))
    assert result.tokens == [int(t) for t in g["tokens"]]
    logits, caches = rt.prefill(prompt, context)
    first = rt.device.argmax(logits)
    logits, caches = rt.decode(first, len(prompt), context, caches)
    assert np.max(np.abs(rt.device.to_numpy(logits) - g["step1_logits"])) <= 2e-2


@pytest.mark.parametrize("name", ["tiny-fp32", "tiny-bf16"])
def test_decode_step_kernel_matches_per_kernel_launches(gpu, name):
    """One cb_decode_step launch per token == the same steps launched one by one."""
    from cuda_b200.compiler import CudaB200Compiler
    from chomikgrad.lazy import register_compiler

    register_compiler("cuda-b200-kernels", lambda: CudaB200Compiler(decode_step=False), replace=True)
    wl = WORKLOADS[name]
    weights = synthetic_weights(wl.config, dtype=wl.np_dtype)
    fused = LlamaRuntime(wl.config, weights, compiler="cuda-b200")
    split = LlamaRuntime(wl.config, weights, compiler="cuda-b200-kernels")
    prompt, context = [5, 17, 3, 99, 42, 7], 64
    logits_a, caches_a = fused.prefill(prompt, context)
    logits_b, caches_b = split.prefill(prompt, context)
    token = fused.device.argmax(logits_a)
    assert token == split.device.argmax(logits_b)
    for i in range(12):  # graph capture from the second run on, for both
        position = len(prompt) + i
        logits_a, caches_a = fused.decode(token, position, context, caches_a)
        logits_b, caches_b = split.decode(token, position, context, caches_b)
        a, b = fused.device.to_numpy(logits_a), split.device.to_numpy(logits_b)
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
        token = fused.device.argmax(logits_a)
        assert token == split.device.argmax(logits_b)
    np.testing.assert_allclose(fused.device.to_numpy(caches_a[-1]), split.device.to_numpy(caches_b[-1]),
                               rtol=1e-5, atol=1e-6)
    program, _ = next(iter(fused._decoders.values()))
    assert program.step_mode and program.launches == 1
    assert not next(iter(split._decoders.values()))[0].step_mode


def test_tiny_bf16_with_every_linear_on_the_tensor_core_gemm(gpu):
    """The prefill Linears on cb_gemm_tc (no row minimum) keep the golden bars."""
    from cuda_b200.compiler import CudaB200Compiler
    from chomikgrad.lazy import register_compiler

    register_compiler("cuda-b200-gemm", lambda: CudaB200Compiler(gemm_min_rows=1), replace=True)
    g = golden("tiny_bf16")
    wl = WORKLOADS["tiny-bf16"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200-gemm")
    logits, _ = rt.prefill(list(g["prompt"]), int(g["context"]))
    program = next(iter(rt._prefill.values()))[0]
    assert program.launches > len(program.plan.steps)  # the float32 activations were split
    assert np.max(np.abs(rt.device.to_numpy(logits) - g["prefill_logits"])) <= 2e-2
    result = rt.generate(list(g["prompt"]), len(g["tokens"]))
    assert result.tokens == [int(t) for t in g["tokens"]]


def test_reference_graphs_through_chomikgrad_compile_graph(gpu):
    """The reference's own entry points with no plugin runtime in between, driven the way
    examples/generate_tinyllama.py:727-857 drives them: chomikgrad.compile_graph(...,
    compiler="cuda-b200", dynamic_inputs=...) of LlamaForCausalLM.prefill and LlamaDecoderStep,
    CompiledProgram.run(bindings), DeviceAdapter.array / argmax; the caches returned by one step
    are bound as the next step's inputs."""
    import chomikgrad
    from chomikgrad import llama as L
    from cuda_b200.graphs import decode_masks

    g = golden("tiny_bf16")
    wl = WORKLOADS["tiny-bf16"]
    cfg, dt = wl.config, wl.np_dtype
    device = chomikgrad.get_compiler("cuda-b200").device
    weights = {}
    for name, value in synthetic_weights(cfg, dtype=dt).items():
        native = device.array(value)
        weights[name] = chomikgrad.Tensor.from_native(native, backend="cuda-b200", shape=tuple(native.shape),
                                                      dtype=device.dtype(native))
    prompt, context = [int(t) for t in g["prompt"]], int(g["context"])
    with chomikgrad.no_grad():
        model = L.LlamaForCausalLM(cfg, weights, sequence_length=len(prompt), dtype=dt, cache_length=context)
        ids = chomikgrad.Tensor(np.asarray([prompt], np.int32), copy=False)
        selector = chomikgrad.Tensor(L.position_selector(len(prompt) - 1, len(prompt), dtype=dt), copy=False)
        prefill = chomikgrad.compile_graph(*model.prefill(ids, selector), compiler="cuda-b200",
                                           dynamic_inputs=(ids,))
    native = prefill.run(None, synchronize=False)
    assert np.max(np.abs(device.to_numpy(native[0]) - g["prefill_logits"])) <= 2e-2
    tokens, caches = [device.argmax(native[0])], list(native[1:])
    step = L.LlamaDecoderStep(cfg, weights, cache_length=context, dtype=dt)
    decoder = nodes = None
    for i in range(1, len(g["tokens"])):
        position = len(prompt) + i - 1
        host = [np.asarray([[tokens[-1]]], np.int32),
                L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=position),
                *decode_masks(position, context, dt), np.asarray(position, np.int32)]
        if decoder is None:
            inputs = [chomikgrad.Tensor(v, copy=False) for v in host]
            cache_inputs = [chomikgrad.Tensor.from_native(c, backend="cuda-b200", shape=tuple(c.shape), dtype=dt)
                            for c in caches]
            with chomikgrad.no_grad():
                outs = step(*inputs[:4], list(zip(cache_inputs[::2], cache_inputs[1::2])), position=inputs[4])
            decoder = chomikgrad.compile_graph(*outs, compiler="cuda-b200", dynamic_inputs=inputs + cache_inputs)
            nodes = [t._node for t in inputs + cache_inputs]
            native = decoder.run(None, synchronize=False)
        else:
            native = decoder.run(dict(zip(nodes, [device.array(v) for v in host] + caches)), synchronize=False)
        tokens.append(device.argmax(native[0]))
        caches = list(native[1:])
    assert tokens == [int(t) for t in g["tokens"]]
