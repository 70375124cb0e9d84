"""Host-side planning (no GPU): views, lowering matches, decode fusion."""

from __future__ import annotations

from collections import Counter
import itertools

import numpy as np
import pytest

from chomikgrad import llama as L
from chomikgrad.tensor import Tensor
from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights
from cuda_b200.graphs import decode_masks
from cuda_b200.planner import Planner, PlanError, reshape_strides


def _leaf_dtype(node):
    if node.value is not None:
        return np.asarray(node.value).dtype
    return np.asarray(next(iter(node.native_values.values()))).dtype


def plan(outputs, dynamic=()):
    return Planner([o._node for o in outputs], [d._node for d in dynamic], backend="cuda-b200",
                   leaf_dtype=_leaf_dtype).build()


def test_reshape_strides_agree_with_numpy():
    rng = np.random.default_rng(0)
    for _ in range(300):
        ndim = rng.integers(1, 5)
        shape = tuple(int(n) for n in rng.integers(1, 5, size=ndim))
        base = np.arange(int(np.prod(shape))).reshape(shape)
        view = base.transpose(rng.permutation(ndim))
        elems = view.size
        # candidate target shapes: factorisations of the size
        factors = [d for d in range(1, elems + 1) if elems % d == 0]
        target = (int(rng.choice(factors)),)
        target = target + (elems // target[0],)
        strides = tuple(s // view.itemsize for s in view.strides)
        got = reshape_strides(view.shape, strides, target)
        try:
            expected = view.view()
            expected.shape = target  # raises when numpy would need a copy
        except AttributeError:
            assert got is None
            continue
        assert got is not None
        # same element addressing
        idx = [np.unravel_index(i, target) for i in range(elems)]
        exp_offsets = [sum(i * s // view.itemsize for i, s in zip(ix, expected.strides)) for ix in idx]
        got_offsets = [sum(i * s for i, s in zip(ix, got)) for ix in idx]
        assert exp_offsets == got_offsets


@pytest.fixture(scope="module")
def tiny_bf16():
    wl = WORKLOADS["tiny-bf16"]
    return wl, {n: Tensor(v) for n, v in synthetic_weights(wl.config, dtype=wl.np_dtype).items()}


def _decode_graph(wl, weights, ctx=48, cache_dtype=np.float32):
    cfg, dt = wl.config, wl.np_dtype
    shape = (1, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor.from_native(np.zeros(shape, cache_dtype), backend="cpu", shape=shape, dtype=dt)
              for _ in range(2 * cfg.num_hidden_layers)]
    am, wm = decode_masks(5, ctx, dt)
    inputs = [Tensor(np.array([[3]], np.int32), copy=False),
              Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=5), copy=False),
              Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(5, np.int32), copy=False)]
    outs = L.LlamaDecoderStep(cfg, weights, cache_length=ctx, dtype=dt)(
        *inputs[:4], list(zip(caches[::2], caches[1::2])), position=inputs[4])
    return outs, inputs + caches


def test_decode_step_is_fully_fused(tiny_bf16):
    wl, weights = tiny_bf16
    outs, dynamic = _decode_graph(wl, weights)
    p = plan(outs, dynamic)
    kinds = Counter(s.name for s in p.steps)
    layers = wl.config.num_hidden_layers
    assert kinds == {"gemv": 4 * layers + 1, "decode_attention": layers}
    assert len(p.aliases) == 2 * layers
    assert 0 in p.argmax_of
    # the rotation input is pruned by the rope lowering: not a program input
    assert dynamic[1]._node not in p.inputs
    # layer-0 norm reads the per-token table (bf16 sequential sum precomputed)
    assert p.init_steps and p.init_steps[0]["name"] == "rms_table"
    assert "rms_norm(gather(" in p.source


def test_decode_fusion_respects_runtime_dtypes(tiny_bf16):
    """bf16 caches make the blend bf16 arithmetic -> generic path, not the f32 kernel."""
    wl, weights = tiny_bf16
    import ml_dtypes

    outs, dynamic = _decode_graph(wl, weights, cache_dtype=ml_dtypes.bfloat16)
    p = plan(outs, dynamic)
    assert "decode_attention" not in Counter(s.name for s in p.steps)


def test_prefill_uses_lowerings(tiny_bf16):
    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    m = L.LlamaForCausalLM(cfg, weights, sequence_length=16, dtype=dt, cache_length=48)
    ids = Tensor(synthetic_prompt(cfg, 16), copy=False)
    outs = m.prefill(ids, Tensor(L.position_selector(15, 16, dtype=dt), copy=False))
    p = plan(outs, [ids])
    layers = cfg.num_hidden_layers
    assert p.lowered == {"rms_norm": 2 * layers + 1, "rope": 2 * layers, "sdpa": layers, "place": 2 * layers}
    # the causal mask (-1e4 above the diagonal, 0 elsewhere) allows tile skipping and mask-free tiles
    assert all(s.args["causal"] == 3 for s in p.steps if s.name == "sdpa")


def test_lowering_is_skipped_when_the_portable_graph_differs():
    x = Tensor(np.ones((1, 4), np.float32))
    w = Tensor(np.ones(4, np.float32))
    out = x / ((x * x).mean(axis=-1, keepdims=True) + 1e-5).sqrt() * w
    out._node.lowering = ("rms_norm", (x._node, w._node), 1e-5)
    assert plan([out]).lowered == {"rms_norm": 1}
    other = x * w  # wrong structure under the same hint
    other._node.lowering = ("rms_norm", (x._node, w._node), 1e-5)
    assert plan([other]).lowered == {}


def test_float64_graph_is_rejected():
    with pytest.raises(PlanError):
        plan([Tensor([1.0, 2.0]) * 2.0])


def test_dynamic_input_must_be_a_leaf_of_the_graph():
    a = Tensor(np.ones(2, np.float32))
    b = Tensor(np.ones(2, np.float32))
    with pytest.raises(ValueError):
        plan([a * 2.0], [b])


def test_prefill_linears_take_the_tensor_core_gemm(tiny_bf16):
    """Every ``x @ W.T`` of a bf16 prefill goes to cb_gemm_tc; nothing else does."""
    from cuda_b200.program import gemm_shape

    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    m = L.LlamaForCausalLM(cfg, weights, sequence_length=16, dtype=dt, cache_length=48)
    ids = Tensor(synthetic_prompt(cfg, 16), copy=False)
    outs = m.prefill(ids, Tensor(L.position_selector(15, 16, dtype=dt), copy=False))
    p = plan(outs, [ids])
    matmuls = [s for s in p.steps if s.name == "matmul"]
    picked = [gemm_shape(s, 1) for s in matmuls]
    h, kv, inter = cfg.hidden_size, cfg.num_key_value_heads * cfg.head_size, cfg.intermediate_size
    per_layer = [(16, h, h, h, h), (16, kv, h, h, h), (16, kv, h, h, h), (16, h, h, h, h),
                 (16, inter, h, h, h), (16, inter, h, h, h), (16, h, inter, inter, inter)]
    assert [x for x in picked if x is not None] == per_layer * cfg.num_hidden_layers
    assert picked.count(None) == 1  # the row selector (float32 right operand)
    assert all(gemm_shape(s, 64) is None for s in matmuls)  # 16 rows: below the default


def test_prefill_gemm_epilogues_are_fused(tiny_bf16):
    """With the tensor-core GEMM in play, q/k/v group, SwiGLU and residual adds fold into GEMMs."""
    from cuda_b200 import _lib

    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    m = L.LlamaForCausalLM(cfg, weights, sequence_length=16, dtype=dt, cache_length=48)
    ids = Tensor(synthetic_prompt(cfg, 16), copy=False)
    outs = m.prefill(ids, Tensor(L.position_selector(15, 16, dtype=dt), copy=False))
    p = Planner([o._node for o in outs], [ids._node], backend="cuda-b200", leaf_dtype=_leaf_dtype,
                gemm_min_rows=16).build()
    multi = [s for s in p.steps if s.name == "matmul_multi"]
    kinds = Counter((s.args["epilogue"], len(s.args["weights"])) for s in multi)
    layers = cfg.num_hidden_layers
    assert kinds[(_lib.GEMM_STORE, 3)] == layers  # q, k, v
    assert kinds[(_lib.GEMM_SWIGLU, 2)] == layers  # gate, up
    # residual adds after O and down; layer 0's first add reads the bf16 embedding, kept apart
    assert kinds[(_lib.GEMM_RESIDUAL, 1)] == 2 * layers - 1
    assert sum(1 for s in p.steps if s.name == "elementwise") == 1
    # the input and post-attention norms are the A prologues of q/k/v and gate/up
    assert sum(1 for s in multi if s.args["x_mode"] == _lib.ROWS_X_RMS) == 2 * layers
    assert sum(1 for s in p.steps if s.name == "rms_norm") == 1  # the final norm (read by the row selector)
    # attention writes token-major rows: the head merge before the O projection is a view
    assert not any(s.name == "copy" for s in p.steps)
    assert all(not s.out.is_contiguous() for s in p.steps if s.name == "sdpa")
    for s in multi:
        if s.args["epilogue"] == _lib.GEMM_RESIDUAL:
            assert s.args["residual"].dtype == np.float32


def test_cache_placement_is_lowered_to_a_column_copy(tiny_bf16):
    """x @ cache_placement (llama.py:411-418) becomes cb_place_columns with the right sources."""
    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    m = L.LlamaForCausalLM(cfg, weights, sequence_length=16, dtype=dt, cache_length=48)
    ids = Tensor(synthetic_prompt(cfg, 16), copy=False)
    outs = m.prefill(ids, Tensor(L.position_selector(15, 16, dtype=dt), copy=False))
    p = plan(outs, [ids])
    places = [s for s in p.steps if s.name == "place"]
    assert len(places) == 2 * cfg.num_hidden_layers
    cols = places[0].args["cols"].host
    assert cols.dtype == np.int32 and list(cols) == list(range(16)) + [-1] * 32
    src = places[0].args["src"]
    assert src.shape == (1, cfg.num_key_value_heads, cfg.head_size, 16)
    assert places[0].out.shape == (1, cfg.num_key_value_heads, cfg.head_size, 48)


def test_placement_match_rejects_other_matrices():
    """Only 0/1 matrices with one 1 per row and at most one per column are copies."""
    from cuda_b200.planner import Planner

    x = Tensor(np.ones((2, 3), np.float32))
    cases = {
        "two ones in a row": np.array([[1, 1], [0, 0], [0, 0]], np.float32),
        "shared column": np.array([[1, 0], [1, 0], [0, 1]], np.float32),
        "not 0/1": np.array([[2, 0], [0, 1], [0, 0]], np.float32),
        "empty row": np.array([[1, 0], [0, 1], [0, 0]], np.float32),
    }
    for name, value in cases.items():
        p = plan([x @ Tensor(value)])
        assert [s.name for s in p.steps] == ["matmul"], name
    perm = np.array([[0, 1, 0, 0], [0, 0, 0, 1], [1, 0, 0, 0]], np.float32)
    p = plan([x @ Tensor(perm)])
    assert [s.name for s in p.steps] == ["place"]
    assert list(p.steps[0].args["cols"].host) == [2, 0, -1, 1]


def test_batched_decode_plan_updates_caches_in_place(tiny_bf16):
    """B sequences in one step: caches bound by pointer, blended in place (cb_kv_write), returned aliased."""
    from cuda_b200.batched import BatchedDecoderStep

    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    b, ctx = 4, 48
    shape = (b, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor.from_native(np.zeros(shape, np.float32), backend="cpu", shape=shape, dtype=dt)
              for _ in range(2 * cfg.num_hidden_layers)]
    am, wm = decode_masks(5, ctx, dt)
    inputs = [Tensor(np.full((b, 1), 3, np.int32), copy=False),
              Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=5), copy=False),
              Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(5, np.int32), copy=False)]
    outs = BatchedDecoderStep(cfg, weights, batch=b, cache_length=ctx, dtype=dt)(
        *inputs[:4], list(zip(caches[::2], caches[1::2])), position=inputs[4])
    p = plan(outs, inputs + caches)
    kinds = Counter(s.name for s in p.steps)
    layers = cfg.num_hidden_layers
    assert kinds["kv_write"] == 2 * layers and kinds["sdpa"] == layers
    assert kinds["matmul"] == 7 * layers + 1
    assert sorted(p.aliases) == list(range(1, 2 * layers + 1))
    for c in caches:
        assert p.input_buffers[c._node].bind == "pointer"
    with pytest.raises(ValueError):
        BatchedDecoderStep(cfg, weights, batch=b, cache_length=ctx, dtype=dt)(
            Tensor(np.zeros((b + 1, 1), np.int32)), *inputs[1:4], list(zip(caches[::2], caches[1::2])))


def test_batched_decode_plan_fuses_into_row_gemms_and_one_attention(tiny_bf16):
    """With the row GEMM in play: per layer q/k/v (+ input norm), one attention kernel for
    RoPE + cache blend + attention, O (+ residual), gate/up (+ norm), down (+ SwiGLU, residual)."""
    from cuda_b200 import _lib
    from cuda_b200.batched import BatchedDecoderStep

    wl, weights = tiny_bf16
    cfg, dt = wl.config, wl.np_dtype
    b, ctx = 4, 48
    shape = (b, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor.from_native(np.zeros(shape, np.float32), backend="cpu", shape=shape, dtype=dt)
              for _ in range(2 * cfg.num_hidden_layers)]
    am, wm = decode_masks(5, ctx, dt)
    inputs = [Tensor(np.full((b, 1), 3, np.int32), copy=False),
              Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=5), copy=False),
              Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(5, np.int32), copy=False)]
    outs = BatchedDecoderStep(cfg, weights, batch=b, cache_length=ctx, dtype=dt)(
        *inputs[:4], list(zip(caches[::2], caches[1::2])), position=inputs[4])
    p = Planner([o._node for o in outs], [t._node for t in inputs + caches], backend="cuda-b200",
                leaf_dtype=_leaf_dtype, gemm_min_rows=64).build()
    kinds = Counter(s.name for s in p.steps)
    layers = cfg.num_hidden_layers
    assert kinds["decode_attention_batched"] == layers
    assert kinds["kv_write"] == kinds["rope"] == kinds["sdpa"] == 0
    # 4 row GEMMs per layer + lm_head; layer 0's O projection reads the bf16 embedding residual, so it
    # is a plain row GEMM and its residual add stays apart
    assert kinds["matmul_rows"] == 4 * layers + 1
    assert kinds["matmul"] == 0 and kinds["elementwise"] == 1
    rows = [s for s in p.steps if s.name == "matmul_rows"]
    assert sum(s.args["x_mode"] == _lib.ROWS_X_RMS for s in rows) == 2 * layers + 1
    assert sum(s.args["x_mode"] == _lib.ROWS_X_SWIGLU for s in rows) == layers
    assert sum(s.args["residual"] is not None for s in rows) == 2 * layers - 1
    for s in p.steps:
        if s.name == "decode_attention_batched":
            assert s.args["k_cache"].buf.bind == "pointer" and s.args["batch"] == b
    assert sorted(p.aliases) == list(range(1, 2 * layers + 1))
