"""Planned programs run by the NumPy plan interpreter against the parity oracle (no GPU).

The planner rewrites the reference's graphs: it fuses the decode step into
GEMVs and one attention kernel per layer, folds RMSNorm / SwiGLU / residual
adds into the tensor-core and row GEMMs, fuses the batched step's RoPE,
cache blends and attention, and lowers tensor-parallel all-reduces.  These
tests execute the resulting plans step by step over the plans' own buffers
and views (``tests/plan_interpreter.py``) and compare every program output
with the oracle's evaluation of the unrewritten graph.  The GPU tests then
only have to show that each kernel computes its step.

Bars: float32 models rtol 1e-4 of the logits' scale; bfloat16 models 2e-2
absolute; argmax tokens equal; caches 1e-4 absolute.
"""

from __future__ import annotations

from collections import Counter

import ml_dtypes
import numpy as np
import pytest

from cuda_b200 import _lib
from cuda_b200 import tensor_parallel as tp
from cuda_b200.batched import BatchedDecoderStep, BatchedPrefill
from chomikgrad import llama as L
from chomikgrad.tensor import Tensor, no_grad
from cuda_b200.models import TINY, WORKLOADS, synthetic_prompt, synthetic_weights
from cuda_b200.planner import Planner
from cuda_b200.graphs import decode_masks
from plan_interpreter import PlanInterpreter, run_ranks

BF16 = np.dtype(ml_dtypes.bfloat16)


def _leaf_dtype(node):
    return np.asarray(node.numpy_value()).dtype


def _plan(outputs, dynamic=(), **kw):
    return Planner([o._node for o in outputs], [d._node for d in dynamic], backend="cuda-b200",
                   leaf_dtype=_leaf_dtype, **kw).build()


def _oracle(outputs):
    from oracle.numpy_compiler import NumpyCompiler

    return [np.asarray(v) for v in NumpyCompiler().compile([o._node for o in outputs]).run()]


def _interpret(outputs, dynamic=(), **kw):
    plan = _plan(outputs, dynamic, **kw)
    it = PlanInterpreter(plan)
    it.run()
    return plan, it, it.outputs()


def _close(got, want, dtype, what=""):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape, what
    assert np.all(np.isfinite(got)), f"{what}: the plan read an unwritten value"
    if np.dtype(dtype) == np.float32:
        scale = max(float(np.abs(want).max()), 1e-30)
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-4 * scale, err_msg=what)
    else:
        np.testing.assert_allclose(got, want, rtol=0, atol=2e-2, err_msg=what)


def _weights(name):
    wl = WORKLOADS[name]
    return wl, {n: Tensor(v) for n, v in synthetic_weights(wl.config, dtype=wl.np_dtype).items()}


def _caches(shape, count, seed):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 1, shape).astype(np.float32) for _ in range(count)]


# ------------------------------------------------------------------ generic path
@pytest.mark.parametrize("dtype", [np.float32, BF16])
def test_generic_steps_match_the_oracle(dtype):
    """Views (permute, reshape), fused elementwise trees, reductions, matmul and gather."""
    rng = np.random.default_rng(4)
    x = Tensor(rng.normal(0, 1, (3, 4, 5)).astype(dtype))
    w = Tensor(rng.normal(0, 1, (5, 6)).astype(dtype))
    table = Tensor(rng.normal(0, 1, (7, 5)).astype(dtype))
    ids = Tensor(np.array([[6, 0, 3]], np.int32))
    y = (x.permute(1, 0, 2) * 2.0 + 1.0).exp().sqrt()
    s = (x * x).sum(axis=-1, keepdims=True)
    m = x.max(axis=1)
    mm = x.reshape(12, 5) @ w
    g = table.gather(ids)
    outs = [y, s, m, mm, g, (x / (s + 1e-3)).relu()]
    _, _, got = _interpret(outs)
    for i, (a, b) in enumerate(zip(got, _oracle(outs))):
        _close(a, b, np.float32 if np.dtype(dtype) == np.float32 else dtype, f"output {i}")
    if np.dtype(dtype) != np.float32:  # bf16 sums are sequential: the same rounding sequence
        np.testing.assert_array_equal(got[1].astype(np.float32), _oracle([s])[0].astype(np.float32))


# ------------------------------------------------------------------ bs-1 decode
def _decode_graph(wl, weights, ctx, position, seed, cache_dtype=np.float32):
    cfg, dt = wl.config, wl.np_dtype
    shape = (1, cfg.num_key_value_heads, ctx, cfg.head_size)
    caches = [Tensor.from_native(c.astype(cache_dtype), backend="cpu", shape=shape, dtype=dt)
              for c in _caches(shape, 2 * cfg.num_hidden_layers, seed)]
    am, wm = decode_masks(position, ctx, dt)
    inputs = [Tensor(np.array([[11]], np.int32), copy=False),
              Tensor(L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=position), copy=False),
              Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(position, np.int32), copy=False)]
    with no_grad():
        outs = L.LlamaDecoderStep(cfg, weights, cache_length=ctx, dtype=dt)(
            *inputs[:4], list(zip(caches[::2], caches[1::2])), position=inputs[4])
    return list(outs), inputs + caches


@pytest.mark.parametrize("name", ["tiny-fp32", "tiny-bf16"])
def test_fused_decode_step_plan_matches_the_oracle(name):
    """GEMVs with RMSNorm prologues (layer 0 through the per-row norm table), fused attention
    with RoPE and the in-place cache blend, SwiGLU / residual epilogues, lm_head + argmax."""
    wl, weights = _weights(name)
    outs, dynamic = _decode_graph(wl, weights, ctx=40, position=17, seed=1)
    want = _oracle(outs)
    plan, it, got = _interpret(outs, dynamic)
    kinds = Counter(s.name for s in plan.steps)
    assert kinds == {"gemv": 4 * wl.config.num_hidden_layers + 1, "decode_attention": wl.config.num_hidden_layers}
    _close(got[0], want[0], wl.np_dtype, "logits")
    assert it.argmax(0) == int(np.argmax(want[0]))
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-4, err_msg=f"cache {i}")


def test_bf16_kv_decode_step_plan_matches_the_oracle():
    """bfloat16-KV mode: the fused decode step reads bfloat16 caches and stores the row it writes
    rounded; against the oracle's graph on the same bfloat16 caches (whose blend keeps the new
    row in float32): logits within the bf16 bar, same argmax, caches within one bf16 rounding."""
    wl, weights = _weights("tiny-bf16")
    outs, dynamic = _decode_graph(wl, weights, ctx=40, position=17, seed=1, cache_dtype=BF16)
    want = _oracle(outs)
    plan, it, got = _interpret(outs, dynamic, kv_bf16=True)
    kinds = Counter(s.name for s in plan.steps)
    assert kinds == {"gemv": 4 * wl.config.num_hidden_layers + 1, "decode_attention": wl.config.num_hidden_layers}
    _close(got[0], want[0], BF16, "logits")
    assert it.argmax(0) == int(np.argmax(want[0]))
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        assert a.dtype == BF16, f"cache {i} stays bfloat16"
        b = np.asarray(b, np.float32)
        # one bfloat16 rounding of values whose float32 sums differ in the last bits: within one bf16 ulp
        np.testing.assert_allclose(np.asarray(a, np.float32), b, rtol=2 ** -7, atol=1e-4, err_msg=f"cache {i}")


def test_bf16_kv_prefill_places_bfloat16_caches():
    wl, weights = _weights("tiny-bf16")
    outs, dynamic = _prefill(wl, weights, seq=16, ctx=24)
    want = _oracle(outs)
    plan, _, got = _interpret(outs, dynamic, kv_bf16=True)
    assert any(st.name == "place" and st.out.dtype == BF16 for st in plan.steps)
    _close(got[0], want[0], BF16, "logits")
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        assert a.dtype == BF16
        np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(b, np.float32), rtol=2 ** -7, atol=1e-4,
                                   err_msg=f"cache {i}")


# ------------------------------------------------------------------ prefill
def _prefill(wl, weights, seq, ctx):
    cfg, dt = wl.config, wl.np_dtype
    ids = Tensor(synthetic_prompt(cfg, seq), copy=False)
    with no_grad():
        m = L.LlamaForCausalLM(cfg, weights, sequence_length=seq, dtype=dt, cache_length=ctx)
        outs = m.prefill(ids, Tensor(L.position_selector(seq - 1, seq, dtype=dt), copy=False))
    return list(outs), [ids]


@pytest.mark.parametrize("name,gemm_min_rows", [("tiny-bf16", 16), ("tiny-bf16", None), ("tiny-fp32", 16)])
def test_prefill_plan_matches_the_oracle(name, gemm_min_rows):
    """With gemm_min_rows=16 the bf16 prefill's GEMMs take q/k/v grouping, the RMSNorm A prologue,
    the SwiGLU and residual epilogues, and attention writes token-major rows."""
    wl, weights = _weights(name)
    outs, dynamic = _prefill(wl, weights, seq=16, ctx=24)
    want = _oracle(outs)
    plan, _, got = _interpret(outs, dynamic, gemm_min_rows=gemm_min_rows)
    fused = Counter(s.name for s in plan.steps)["matmul_multi"]
    assert (fused > 0) == (gemm_min_rows is not None and wl.np_dtype != np.float32)
    _close(got[0], want[0], wl.np_dtype, "logits")
    assert int(np.argmax(got[0])) == int(np.argmax(want[0]))
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-4 * max(1.0, float(np.abs(b).max())), err_msg=f"cache {i}")


# ------------------------------------------------------------------ batched decode
def _batched_graph(config, weights, dt, batch, ctx, position, seed, cache_dtype=np.float32):
    shape = (batch, config.num_key_value_heads, ctx, config.head_size)
    caches = [Tensor.from_native(c.astype(cache_dtype), backend="cpu", shape=shape, dtype=dt)
              for c in _caches(shape, 2 * config.num_hidden_layers, seed)]
    am, wm = decode_masks(position, ctx, dt)
    rng = np.random.default_rng(seed)
    inputs = [Tensor(rng.integers(0, config.vocab_size, (batch, 1)).astype(np.int32), copy=False),
              Tensor(L._rope_rotations(1, config.head_size, config.rope_theta, dt, offset=position), copy=False),
              Tensor(am, copy=False), Tensor(wm, copy=False), Tensor(np.asarray(position, np.int32), copy=False)]
    with no_grad():
        outs = BatchedDecoderStep(config, weights, batch=batch, cache_length=ctx, dtype=dt)(
            *inputs[:4], list(zip(caches[::2], caches[1::2])), position=inputs[4])
    return list(outs), inputs + caches


@pytest.mark.parametrize("name", ["tiny-bf16", "tiny-fp32"])
def test_batched_decode_plan_matches_the_oracle(name):
    """bf16: row GEMMs with norm / SwiGLU prologues and residual epilogues, and RoPE + cache
    blends + attention as one step per layer.  float32: the generic kv_write / rope / sdpa path."""
    wl, weights = _weights(name)
    outs, dynamic = _batched_graph(wl.config, weights, wl.np_dtype, batch=3, ctx=40, position=21, seed=2)
    want = _oracle(outs)
    plan, _, got = _interpret(outs, dynamic, gemm_min_rows=64)
    kinds = Counter(s.name for s in plan.steps)
    layers = wl.config.num_hidden_layers
    if wl.np_dtype == np.float32:
        assert kinds["kv_write"] == 2 * layers and kinds["sdpa"] == layers
    else:
        # layer 0's O projection keeps its residual add apart (the residual is the bf16 embedding row)
        assert kinds["decode_attention_batched"] == layers and kinds["matmul_rows"] == 4 * layers + 1
        assert kinds["matmul"] == 0  # nothing left on the SIMT matmul
    _close(got[0], want[0], wl.np_dtype, "logits")
    assert (np.argmax(got[0], -1) == np.argmax(want[0], -1)).all()
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-4, err_msg=f"cache {i}")


def test_bf16_kv_batched_decode_plan_matches_the_oracle():
    wl, weights = _weights("tiny-bf16")
    outs, dynamic = _batched_graph(wl.config, weights, wl.np_dtype, batch=3, ctx=40, position=21, seed=2,
                                   cache_dtype=BF16)
    want = _oracle(outs)
    plan, _, got = _interpret(outs, dynamic, gemm_min_rows=64, kv_bf16=True)
    assert Counter(s.name for s in plan.steps)["decode_attention_batched"] == wl.config.num_hidden_layers
    _close(got[0], want[0], BF16, "logits")
    assert (np.argmax(got[0], -1) == np.argmax(want[0], -1)).all()
    for i, (a, b) in enumerate(zip(got[1:], want[1:])):
        assert a.dtype == BF16
        np.testing.assert_allclose(np.asarray(a, np.float32), np.asarray(b, np.float32), rtol=2 ** -7, atol=1e-4,
                                   err_msg=f"cache {i}")


# ------------------------------------------------------------------ tensor parallel
@pytest.mark.parametrize("size,vocab_shard", [(2, False), (4, False), (2, True), (4, True)])
def test_tensor_parallel_plans_match_the_one_rank_oracle(size, vocab_shard):
    """Each rank's planned batched step (row GEMMs, fused attention, all_reduce steps after O and
    down), run in lock step with the collectives summing the ranks' operands, gives the
    unsharded graph's logits on every rank -- with a vocabulary-sharded lm_head the rank's
    columns of them, no gather in the step -- and the rank's KV heads of its caches."""
    config, batch, ctx, position = TINY, 3, 24, 9
    full_w = {k: v.astype(BF16) for k, v in synthetic_weights(config, dtype=np.float32).items()}
    outs, _ = _batched_graph(config, {k: Tensor(v) for k, v in full_w.items()}, BF16, batch, ctx, position, seed=5)
    want = _oracle(outs)
    full_caches = [np.asarray(c) for c in _caches((batch, config.num_key_value_heads, ctx, config.head_size),
                                                  2 * config.num_hidden_layers, 5)]
    rng = np.random.default_rng(5)
    ids = rng.integers(0, config.vocab_size, (batch, 1)).astype(np.int32)
    am, wm = decode_masks(position, ctx, BF16)
    interpreters, layouts = [], []
    for rank in range(size):
        lay = tp.shard_layout(config, size, rank, vocab_shard=vocab_shard)
        kv = lay.kv_rows.start // config.head_size
        with no_grad():
            step = tp.TensorParallelDecoderStep(
                config, {k: Tensor(v) for k, v in tp.shard_weights(config, full_w, lay).items()}, lay,
                batch=batch, cache_length=ctx, dtype=BF16)
            t = [Tensor(ids), Tensor(L._rope_rotations(1, config.head_size, config.rope_theta, BF16, offset=position)),
                 Tensor(am), Tensor(wm), Tensor(np.asarray(position, np.int32))]
            ct = [Tensor(c[:, kv:kv + lay.kv_heads].copy()) for c in full_caches]
            rank_outs = step(t[0], t[1], t[2], t[3], list(zip(ct[::2], ct[1::2])), position=t[4])
        plan = _plan(list(rank_outs), t + ct, gemm_min_rows=64)
        kinds = Counter(s.name for s in plan.steps)
        assert kinds["all_reduce"] == 2 * config.num_hidden_layers
        assert kinds["decode_attention_batched"] == config.num_hidden_layers
        assert kinds["all_gather"] == 0  # the distributed argmax exchanges records, not logits
        interpreters.append(PlanInterpreter(plan))
        layouts.append((lay, kv))
    run_ranks(interpreters)
    for it, (lay, kv) in zip(interpreters, layouts):
        got = it.outputs()
        columns = lay.vocab_rows if vocab_shard else slice(None)
        _close(got[0], want[0][:, columns], BF16, "logits")
        if not vocab_shard:
            assert (np.argmax(got[0], -1) == np.argmax(want[0], -1)).all()
        for i, (a, b) in enumerate(zip(got[1:], want[1:])):
            np.testing.assert_allclose(a, b[:, kv:kv + lay.kv_heads], rtol=0, atol=1e-4, err_msg=f"cache {i}")


@pytest.mark.parametrize("vocab_shard", [False, True])
def test_tensor_parallel_prefill_plans_match_the_one_rank_oracle(vocab_shard):
    """Each rank's planned prefill (grouped q/k/v, RMSNorm prologues, SwiGLU epilogue on the
    tensor-core GEMM, token-major attention, all_reduce steps after O and down) gives the
    unsharded prefill's logits on every rank and the rank's KV heads of its caches."""
    config, size, seq, ctx = TINY, 2, 16, 24
    full_w = {k: v.astype(BF16) for k, v in synthetic_weights(config, dtype=np.float32).items()}
    ids = np.random.default_rng(3).integers(0, config.vocab_size, (1, seq)).astype(np.int32)
    selector = L.position_selector(seq - 1, seq, dtype=BF16)
    with no_grad():
        model = L.LlamaForCausalLM(config, {k: Tensor(v) for k, v in full_w.items()}, sequence_length=seq,
                                   dtype=BF16, cache_length=ctx)
        want = _oracle(list(model.prefill(Tensor(ids), Tensor(selector))))
    interpreters, layouts = [], []
    for rank in range(size):
        lay = tp.shard_layout(config, size, rank, vocab_shard=vocab_shard)
        with no_grad():
            m = tp.TensorParallelPrefill(config, {k: Tensor(v) for k, v in tp.shard_weights(config, full_w, lay).items()},
                                         lay, sequence_length=seq, dtype=BF16, cache_length=ctx)
            source = Tensor(ids)
            outs = list(m.prefill(source, Tensor(selector)))
        plan = _plan(outs, [source], gemm_min_rows=16)
        kinds = Counter(s.name for s in plan.steps)
        assert kinds["all_reduce"] == 2 * config.num_hidden_layers and kinds["matmul_multi"] > 0
        assert kinds["all_gather"] == int(vocab_shard)  # the prefill returns the whole logits
        interpreters.append(PlanInterpreter(plan))
        layouts.append((lay, lay.kv_rows.start // config.head_size))
    run_ranks(interpreters)
    for it, (lay, kv) in zip(interpreters, layouts):
        got = it.outputs()
        _close(got[0], want[0], BF16, "logits")
        assert int(np.argmax(got[0])) == int(np.argmax(want[0]))
        for i, (a, b) in enumerate(zip(got[1:], want[1:])):
            b = np.asarray(b, np.float32)[:, kv:kv + lay.kv_heads]
            np.testing.assert_allclose(a, b, rtol=0, atol=1e-4 * max(1.0, float(np.abs(b).max())), err_msg=f"cache {i}")


# ------------------------------------------------------------------ batched prefill
@pytest.mark.parametrize("name", ["tiny-bf16", "tiny-fp32"])
def test_batched_prefill_plan_matches_each_prompts_prefill(name):
    """BatchedPrefill (three prompts as one graph, every Linear a GEMM over all rows): the
    planned program gives each prompt's batch-1 prefill -- the oracle's logits and caches of the
    reference's LlamaForCausalLM run on that prompt alone."""
    wl, weights = _weights(name)
    cfg, dt = wl.config, wl.np_dtype
    b, seq, ctx = 3, 16, 24
    ids = np.concatenate([synthetic_prompt(cfg, seq, seed=s) for s in range(b)]).astype(np.int32)
    selector = L.position_selector(seq - 1, seq, dtype=dt)
    with no_grad():
        source = Tensor(ids, copy=False)
        outs = list(BatchedPrefill(cfg, weights, batch=b, sequence_length=seq, dtype=dt,
                                   cache_length=ctx).prefill(source, Tensor(selector, copy=False)))
    plan, _, got = _interpret(outs, [source], gemm_min_rows=16)
    assert got[0].shape == (b, cfg.vocab_size)
    for s in range(b):
        with no_grad():
            one = L.LlamaForCausalLM(cfg, weights, sequence_length=seq, dtype=dt, cache_length=ctx)
            want = _oracle(list(one.prefill(Tensor(ids[s:s + 1], copy=False), Tensor(selector, copy=False))))
        _close(got[0][s:s + 1], want[0], dt, f"logits of prompt {s}")
        assert int(np.argmax(got[0][s])) == int(np.argmax(want[0]))
        for i, (a, w) in enumerate(zip(got[1:], want[1:])):
            w = np.asarray(w, np.float32)
            np.testing.assert_allclose(np.asarray(a, np.float32)[s:s + 1], w, rtol=0,
                                       atol=1e-4 * max(1.0, float(np.abs(w).max())), err_msg=f"prompt {s} cache {i}")


def test_tensor_parallel_batched_prefill_plans_match_the_one_rank_oracle():
    """Two ranks' batched prefills (two prompts): every rank's logits are the unsharded batch-1
    prefill's, prompt by prompt, and its caches are its KV heads of that prompt's caches."""
    config, size, b, seq, ctx = TINY, 2, 2, 16, 24
    full_w = {k: v.astype(BF16) for k, v in synthetic_weights(config, dtype=np.float32).items()}
    ids = np.random.default_rng(5).integers(0, config.vocab_size, (b, seq)).astype(np.int32)
    selector = L.position_selector(seq - 1, seq, dtype=BF16)
    wants = []
    for s in range(b):
        with no_grad():
            model = L.LlamaForCausalLM(config, {k: Tensor(v) for k, v in full_w.items()}, sequence_length=seq,
                                       dtype=BF16, cache_length=ctx)
            wants.append(_oracle(list(model.prefill(Tensor(ids[s:s + 1]), Tensor(selector)))))
    interpreters, layouts = [], []
    for rank in range(size):
        lay = tp.shard_layout(config, size, rank, vocab_shard=True)
        with no_grad():
            m = tp.TensorParallelBatchedPrefill(
                config, {k: Tensor(v) for k, v in tp.shard_weights(config, full_w, lay).items()}, lay, batch=b,
                sequence_length=seq, dtype=BF16, cache_length=ctx)
            source = Tensor(ids)
            outs = list(m.prefill(source, Tensor(selector)))
        plan = _plan(outs, [source], gemm_min_rows=16)
        kinds = Counter(s.name for s in plan.steps)
        assert kinds["all_reduce"] == 2 * config.num_hidden_layers and kinds["all_gather"] == 1
        interpreters.append(PlanInterpreter(plan))
        layouts.append((lay, lay.kv_rows.start // config.head_size))
    run_ranks(interpreters)
    for it, (lay, kv) in zip(interpreters, layouts):
        got = it.outputs()
        for s, want in enumerate(wants):
            _close(got[0][s:s + 1], want[0], BF16, f"logits of prompt {s}")
            assert int(np.argmax(got[0][s])) == int(np.argmax(want[0]))
            for i, (a, w) in enumerate(zip(got[1:], want[1:])):
                w = np.asarray(w, np.float32)[:, kv:kv + lay.kv_heads]
                np.testing.assert_allclose(np.asarray(a, np.float32)[s:s + 1], w, rtol=0,
                                           atol=1e-4 * max(1.0, float(np.abs(w).max())), err_msg=f"cache {i}")


# ------------------------------------------------------------------ the interpreter itself
def test_interpreter_catches_a_wrong_operand():
    """A plan whose fused step reads the wrong buffer is caught (the check has teeth)."""
    wl, weights = _weights("tiny-fp32")
    outs, dynamic = _decode_graph(wl, weights, ctx=40, position=17, seed=1)
    want = _oracle(outs)
    plan = _plan(outs, dynamic)
    gemvs = [s for s in plan.steps if s.name == "gemv" and s.args["epilogue"] == _lib.EPI_RESIDUAL]
    first, second = gemvs[1], gemvs[2]
    first.args["residual"], second.args["residual"] = second.args["residual"], first.args["residual"]
    it = PlanInterpreter(plan)
    it.run()
    got = it.outputs()[0]
    assert not np.allclose(got, want[0], rtol=0, atol=1e-4 * float(np.abs(want[0]).max()))
