"""The plugin under the unmodified reference package (no GPU needed).

``cuda_b200`` registers ``cuda-b200`` in ``chomikgrad``'s own registry and
its classes are the reference's plugin ABCs' subclasses.  The graphs here are
built by the reference's ``chomikgrad.llama`` (``LlamaForCausalLM.prefill``,
``LlamaDecoderStep``, ``LlamaDecoderBlock``), planned by the plugin's
``Planner`` and executed step by step by ``tests/plan_interpreter.py``; the
comparison is against the reference's OWN ``NumpyCompiler``
(chomikgrad/lazy.py:551-636) on the same graphs, and the restated oracle is
checked bit for bit against that compiler as well.
"""

from __future__ import annotations

from collections import Counter

import numpy as np
import pytest

import chomikgrad
from chomikgrad import llama as L
from chomikgrad.lazy import NumpyCompiler as ReferenceCompiler
from chomikgrad.tensor import Tensor, no_grad
import cuda_b200
from cuda_b200.graphs import decode_masks
from cuda_b200.models import TINYLLAMA, WORKLOADS, synthetic_prompt, synthetic_weights
from cuda_b200.planner import Planner
from plan_interpreter import PlanInterpreter


def _reference(outputs):
    return [np.asarray(v) for v in ReferenceCompiler().compile([o._node for o in outputs]).run()]


def _leaf_dtype(node):
    return np.asarray(node.numpy_value()).dtype


def test_plugin_is_registered_in_the_reference_registry():
    from cuda_b200.compiler import CudaB200Compiler
    from cuda_b200.device import CudaB200Device
    from cuda_b200.program import CudaB200Program

    assert cuda_b200.BACKEND in chomikgrad.lazy._COMPILERS
    assert issubclass(CudaB200Compiler, chomikgrad.Compiler)
    assert issubclass(CudaB200Device, chomikgrad.DeviceAdapter)
    assert issubclass(CudaB200Program, chomikgrad.CompiledProgram)
    cuda_b200.install()  # idempotent (replace)
    with pytest.raises(ValueError):
        cuda_b200.install(replace=False)


def _graphs(name, seed=3):
    """Reference-built prefill, decode step and 3-token verify block of a tiny model."""
    wl = WORKLOADS[name]
    cfg, dt = wl.config, wl.np_dtype
    weights = {n: Tensor(v) for n, v in synthetic_weights(cfg, dtype=dt).items()}
    seq, ctx, pos = 9, 24, 13
    rng = np.random.default_rng(seed)
    shape = (1, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor(rng.normal(0, 1, shape).astype(np.float32)) for _ in range(2 * cfg.num_hidden_layers)]
    with no_grad():
        ids = Tensor(synthetic_prompt(cfg, seq), copy=False)
        prefill = L.LlamaForCausalLM(cfg, weights, sequence_length=seq, dtype=dt, cache_length=ctx).prefill(
            ids, Tensor(L.position_selector(seq - 1, seq, dtype=dt), copy=False))
        am, wm = decode_masks(pos, ctx, dt)
        step_in = [Tensor(np.array([[21]], np.int32), copy=False),
                   Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=pos), copy=False),
                   Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(pos, np.int32), copy=False)]
        decode = L.LlamaDecoderStep(cfg, weights, cache_length=ctx, dtype=dt)(
            *step_in[:4], list(zip(caches[::2], caches[1::2])), position=step_in[4])
        t = 3
        placement = np.zeros((t, ctx), dt)
        placement[np.arange(t), pos + np.arange(t)] = 1
        mask = np.full((1, 1, t, ctx), -1e4, dt)
        for i in range(t):
            mask[0, 0, i, : pos + i + 1] = 0
        block = L.LlamaDecoderBlock(cfg, weights, block_length=t, cache_length=ctx, dtype=dt)(
            Tensor(np.array([[5, 6, 7]], np.int32), copy=False),
            Tensor(L._rope_rotations(t, cfg.head_size, cfg.rope_theta, dt, offset=pos)),
            Tensor(mask), Tensor(placement), Tensor(placement.sum(axis=0).reshape(1, 1, ctx, 1)),
            list(zip(caches[::2], caches[1::2])))
    return wl, {"prefill": (list(prefill), [ids]), "decode": (list(decode), step_in + caches),
                "block": (list(block), [])}


@pytest.mark.parametrize("name", ["tiny-fp32", "tiny-bf16"])
def test_oracle_equals_the_reference_compiler_bit_for_bit(oracle, name):
    _, graphs = _graphs(name)
    for kind, (outs, _) in graphs.items():
        want = _reference(outs)
        got = [np.asarray(v) for v in oracle.NumpyCompiler().compile([o._node for o in outs]).run()]
        for i, (a, b) in enumerate(zip(got, want)):
            assert a.dtype == b.dtype and np.array_equal(a, b, equal_nan=True), f"{kind} output {i}"


@pytest.mark.parametrize("name", ["tiny-fp32", "tiny-bf16"])
def test_planned_reference_graphs_match_the_reference_compiler(name):
    """Prefill (tensor-core GEMM fusions from 8 rows), the fused decode step and the verify
    block, planned from the reference's own graphs, against the reference's own compiler."""
    wl, graphs = _graphs(name)
    for kind, (outs, dynamic) in graphs.items():
        want = _reference(outs)
        plan = Planner([o._node for o in outs], [d._node for d in dynamic], backend=cuda_b200.BACKEND,
                       leaf_dtype=_leaf_dtype, gemm_min_rows=8).build()
        it = PlanInterpreter(plan)
        it.run()
        got = it.outputs()
        scale = float(np.abs(want[0]).max())
        if wl.np_dtype == np.float32:
            np.testing.assert_allclose(got[0], want[0], rtol=0, atol=1e-4 * scale, err_msg=kind)
        else:
            np.testing.assert_allclose(np.asarray(got[0], np.float32), np.asarray(want[0], np.float32),
                                       rtol=0, atol=2e-2, err_msg=kind)
        assert (np.argmax(got[0], -1) == np.argmax(want[0], -1)).all(), kind
        for i, (a, b) in enumerate(zip(got[1:], want[1:])):
            b = np.asarray(b, np.float32)
            np.testing.assert_allclose(np.asarray(a, np.float32), b, rtol=0,
                                       atol=1e-4 * max(1.0, float(np.abs(b).max())), err_msg=f"{kind} cache {i}")
        if kind == "decode":
            kinds = Counter(s.name for s in plan.steps)
            layers = wl.config.num_hidden_layers
            assert kinds == {"gemv": 4 * layers + 1, "decode_attention": layers}


def test_tinyllama_reference_decode_graph_plans_into_the_fused_step():
    """The reference's TinyLlama-shape LlamaDecoderStep (22 layers) plans into 89 GEMVs and 22
    fused attention steps -- the phases of the one cb_decode_step launch (planning only)."""
    import ml_dtypes

    cfg, dt, ctx, pos = TINYLLAMA, np.dtype(ml_dtypes.bfloat16), 384, 200
    shapes = L.required_weight_shapes(cfg)
    weights = {n: Tensor.from_native(np.zeros(1, dt), backend="placeholder", shape=s, dtype=dt)
               for n, s in shapes.items()}
    shape = (1, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor.from_native(np.zeros(1, dt), backend="placeholder", shape=shape, dtype=dt)
              for _ in range(2 * cfg.num_hidden_layers)]
    am, wm = decode_masks(pos, ctx, dt)
    step_in = [Tensor(np.array([[21]], np.int32), copy=False),
               Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=pos), copy=False),
               Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(pos, np.int32), copy=False)]
    with no_grad():
        outs = L.LlamaDecoderStep(cfg, weights, cache_length=ctx, dtype=dt)(
            *step_in[:4], list(zip(caches[::2], caches[1::2])), position=step_in[4])

    def leaf_dtype(node):
        return np.dtype(np.float32) if any(node is c._node for c in caches) else node.dtype

    plan = Planner([o._node for o in outs], [d._node for d in step_in + caches], backend=cuda_b200.BACKEND,
                   leaf_dtype=leaf_dtype).build()
    kinds = Counter(s.name for s in plan.steps)
    assert kinds == {"gemv": 4 * cfg.num_hidden_layers + 1, "decode_attention": cfg.num_hidden_layers}
