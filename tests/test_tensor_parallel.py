"""Tensor-parallel graphs on the CPU: sharding, planning, and equality with the one-rank graph.

Each rank's graph (cuda_b200.tensor_parallel) runs on the parity oracle, with
its ``all_reduce`` nodes summing the ranks' partials: ranks are threads of one
process (a barrier and a rank-ordered sum) or, in the last test, two
processes over torch.distributed's gloo backend.  The logits and caches must
equal the unsharded graph's up to float32 reassociation of the row-sharded
sums (the O and down projections add G partial dot products).
"""

from __future__ import annotations

import threading
from typing import Callable, Dict, List

import numpy as np
import pytest

from cuda_b200 import tensor_parallel as tp
from cuda_b200.batched import BatchedDecoderStep
from chomikgrad.llama import LlamaForCausalLM, _rope_rotations as rope_rotations, position_selector
from cuda_b200.graphs import decode_masks
from chomikgrad.lazy import topological_sort
from chomikgrad.tensor import Tensor, no_grad
from cuda_b200.models import LLAMA3_8B, TINY, TINYLLAMA, synthetic_weights
from cuda_b200.planner import Planner
from oracle.numpy_compiler import evaluate_node


def test_layouts_of_the_benchmark_shapes():
    for size in (1, 2, 4, 8):
        for rank in range(size):
            lay = tp.shard_layout(LLAMA3_8B, size, rank)
            assert (lay.heads, lay.kv_heads, lay.intermediate) == (32 // size, 8 // size, 14336 // size)
            assert lay.kv_start == rank * lay.kv_heads * 128 and lay.group == 4
    # TinyLlama on 8 ranks: 4 KV heads, each replicated on two ranks
    starts = [tp.shard_layout(TINYLLAMA, 8, r).kv_start // 64 for r in range(8)]
    assert starts == [0, 0, 1, 1, 2, 2, 3, 3]
    with pytest.raises(ValueError):
        tp.shard_layout(TINYLLAMA, 3, 0)


def test_shards_reassemble_the_weights():
    weights = synthetic_weights(TINY, dtype=np.float32)
    shards = [tp.shard_weights(TINY, weights, tp.shard_layout(TINY, 2, r)) for r in range(2)]
    for name, w in weights.items():
        parts = [s[name] for s in shards]
        if name.endswith(("o_proj.weight", "down_proj.weight")):
            np.testing.assert_array_equal(np.concatenate(parts, axis=1), w)
        elif name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight",
                            "up_proj.weight")):
            np.testing.assert_array_equal(np.concatenate(parts, axis=0), w)
        else:
            assert all(p is w for p in parts)


# ---------------------------------------------------------------- graphs
def _tensors(weights):
    return {k: Tensor(v) for k, v in weights.items()}


def _decode_inputs(config, batch, context, position, seed):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, config.vocab_size, (batch, 1)).astype(np.int32)
    rotation = rope_rotations(1, config.head_size, config.rope_theta, np.float32, offset=position)
    attention, write = decode_masks(position, context, np.float32)
    shape = (batch, config.num_key_value_heads, context, config.head_size)
    caches = [rng.normal(0, 1, shape).astype(np.float32) for _ in range(2 * config.num_hidden_layers)]
    return ids, rotation, attention, write, np.asarray(position, np.int32), caches


def _tp_decode_graph(config, weights, layout, batch, context, inputs):
    """One rank's decode step over its shards and its KV heads of the caches."""
    ids, rotation, attention, write, position, caches = inputs
    kv = layout.kv_rows.start // config.head_size
    local = [c[:, kv:kv + layout.kv_heads] for c in caches]
    with no_grad():
        step = tp.TensorParallelDecoderStep(config, _tensors(tp.shard_weights(config, weights, layout)), layout,
                                            batch=batch, cache_length=context, dtype=np.float32)
        t = [Tensor(v) for v in (ids, rotation, attention, write, position)]
        ct = [Tensor(c) for c in local]
        return step(t[0], t[1], t[2], t[3], list(zip(ct[::2], ct[1::2])), position=t[4])


def _run(outputs, reduce_fn: Callable[[np.ndarray], np.ndarray],
         gather_fn: Callable[[np.ndarray], np.ndarray] = None) -> List[np.ndarray]:
    """The oracle's evaluation, with all_reduce / all_gather nodes computed by ``reduce_fn`` / ``gather_fn``."""
    nodes = [o._node for o in outputs]
    values: Dict[object, np.ndarray] = {}
    for node in topological_sort(nodes):
        if node.op is None:
            values[node] = node.numpy_value()
        elif node.lowering is not None and node.lowering[0] == "all_reduce":
            values[node] = reduce_fn(values[node.lowering[1][0]])
        elif node.lowering is not None and node.lowering[0] == "all_gather" and gather_fn is not None:
            values[node] = gather_fn(values[node.lowering[1][0]])
        else:
            values[node] = evaluate_node(node, [values[p] for p in node.inputs])
    return [np.asarray(values[n]) for n in nodes]


def _threaded_ranks(size: int, build: Callable[[int], list]) -> List[List[np.ndarray]]:
    """Evaluate every rank's graph on its own thread; all_reduce sums in rank order."""
    barrier = threading.Barrier(size)
    slots: List = [None] * size
    results: List = [None] * size
    errors: List = []

    # graphs are built here, one rank after another: the reference's grad mode
    # (no_grad) is a process-wide flag that concurrent builders would leave off
    built = [build(rank) for rank in range(size)]

    def worker(rank: int) -> None:
        try:
            outputs = built[rank]

            def reduce_fn(x):
                slots[rank] = x
                barrier.wait(timeout=60)
                total = slots[0].astype(np.float32)
                for other in slots[1:]:
                    total = total + other
                barrier.wait(timeout=60)
                return total.astype(x.dtype)

            def gather_fn(x):
                slots[rank] = x
                barrier.wait(timeout=60)
                stacked = np.stack([np.asarray(v) for v in slots])
                barrier.wait(timeout=60)
                return stacked.astype(x.dtype)

            results[rank] = _run(outputs, reduce_fn, gather_fn)
        except Exception as exc:  # noqa: BLE001
            errors.append(exc)
            barrier.abort()

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(size)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    if errors:
        raise errors[0]
    return results


@pytest.mark.parametrize("size", [2, 4])
def test_tensor_parallel_decode_equals_one_rank(size):
    config, batch, context, position = TINY, 3, 24, 9
    weights = synthetic_weights(config, dtype=np.float32)
    inputs = _decode_inputs(config, batch, context, position, seed=size)
    ids, rotation, attention, write, pos, caches = inputs
    with no_grad():
        step = BatchedDecoderStep(config, _tensors(weights), batch=batch, cache_length=context, dtype=np.float32)
        t = [Tensor(v) for v in (ids, rotation, attention, write, pos)]
        ct = [Tensor(c) for c in caches]
        full = _run(step(t[0], t[1], t[2], t[3], list(zip(ct[::2], ct[1::2])), position=t[4]), lambda x: x)
    ranks = _threaded_ranks(size, lambda r: _tp_decode_graph(config, weights, tp.shard_layout(config, size, r),
                                                             batch, context, inputs))
    scale = float(np.abs(full[0]).max())
    for rank, got in enumerate(ranks):
        lay = tp.shard_layout(config, size, rank)
        np.testing.assert_allclose(got[0], full[0], rtol=0, atol=1e-4 * scale)  # logits on every rank
        assert (got[0].argmax(-1) == full[0].argmax(-1)).all()
        kv = lay.kv_rows.start // config.head_size
        for g, f in zip(got[1:], full[1:]):  # the rank's KV heads of the updated caches
            np.testing.assert_allclose(g, f[:, kv:kv + lay.kv_heads], rtol=0, atol=1e-5)


def _pick(records):
    """The distributed argmax's pick (cb_argmax_pick): records (ranks, rows, [value, global index]) in rank
    order -> per row a NaN first, then the larger value, then the lower index."""
    out = []
    for row in range(records.shape[1]):
        best = None
        for value, index in records[:, row]:
            if best is None:
                best = (value, index)
                continue
            bv, bi = best
            if np.isnan(value) or np.isnan(bv):
                better = np.isnan(value) and (not np.isnan(bv) or index < bi)
            else:
                better = value > bv or (value == bv and index < bi)
            if better:
                best = (value, index)
        out.append(int(best[1]))
    return np.asarray(out)


def _records(local, offset):
    """One rank's records: np.argmax of its columns, as a global index."""
    idx = np.argmax(local, axis=-1)
    return np.stack([local[np.arange(local.shape[0]), idx], idx + offset], axis=-1)


@pytest.mark.parametrize("size", [2, 4])
def test_distributed_argmax_equals_argmax_of_the_whole_row(size):
    rng = np.random.default_rng(size)
    vocab = 64 * size
    logits = rng.normal(0, 1, (9, vocab)).astype(np.float32)
    logits[1, [5, 64]] = 9.0                       # a tie across a shard boundary: the lower index wins
    logits[2, [vocab - 1, 0]] = 7.0
    logits[3, 70] = np.nan                         # NaN wins wherever it is
    logits[4, [3, vocab - 2]] = np.nan             # the first NaN wins
    logits[5] = 0.0                                # all equal: index 0
    logits[6, -1] = np.inf
    logits[7] = -np.inf
    logits[8, [10, 10 + vocab // size]] = np.finfo(np.float32).max
    cols = vocab // size
    records = np.stack([_records(logits[:, r * cols:(r + 1) * cols], r * cols) for r in range(size)])
    np.testing.assert_array_equal(_pick(records), np.argmax(logits, axis=-1))


@pytest.mark.parametrize("size", [2, 4])
def test_vocabulary_sharded_lm_head_returns_the_rank_columns(size):
    """With the lm_head's rows split over the ranks, each rank's decode step returns its columns of the
    unsharded logits, and the records of the distributed argmax pick the unsharded greedy tokens."""
    config, batch, context, position = TINY, 3, 24, 9
    weights = synthetic_weights(config, dtype=np.float32)
    inputs = _decode_inputs(config, batch, context, position, seed=11)
    ids, rotation, attention, write, pos, caches = inputs
    with no_grad():
        step = BatchedDecoderStep(config, _tensors(weights), batch=batch, cache_length=context, dtype=np.float32)
        t = [Tensor(v) for v in (ids, rotation, attention, write, pos)]
        ct = [Tensor(c) for c in caches]
        full = _run(step(t[0], t[1], t[2], t[3], list(zip(ct[::2], ct[1::2])), position=t[4]), lambda x: x)
    layouts = [tp.shard_layout(config, size, r, vocab_shard=True) for r in range(size)]
    assert sum(lay.vocab for lay in layouts) == config.vocab_size
    assert tp.shard_weights(config, weights, layouts[1])["lm_head.weight"].shape[0] == config.vocab_size // size
    ranks = _threaded_ranks(size, lambda r: _tp_decode_graph(config, weights, layouts[r], batch, context, inputs))
    scale = float(np.abs(full[0]).max())
    for lay, got in zip(layouts, ranks):
        np.testing.assert_allclose(got[0], full[0][:, lay.vocab_rows], rtol=0, atol=1e-4 * scale)
    records = np.stack([_records(got[0], lay.vocab_start) for lay, got in zip(layouts, ranks)])
    np.testing.assert_array_equal(_pick(records), full[0].argmax(-1))
    import dataclasses

    with pytest.raises(ValueError, match="vocabulary"):
        tp.shard_layout(dataclasses.replace(config, vocab_size=4095), 2, 0, vocab_shard=True)


def test_tensor_parallel_prefill_equals_one_rank():
    config, size, seq, context = TINY, 2, 12, 20
    weights = synthetic_weights(config, dtype=np.float32)
    ids = np.random.default_rng(3).integers(0, config.vocab_size, (1, seq)).astype(np.int32)
    selector = position_selector(seq - 1, seq, dtype=np.float32)
    with no_grad():
        model = LlamaForCausalLM(config, _tensors(weights), sequence_length=seq, dtype=np.float32,
                                 cache_length=context)
        full = _run(model.prefill(Tensor(ids), Tensor(selector)), lambda x: x)

    def build(rank):
        lay = tp.shard_layout(config, size, rank)
        with no_grad():
            m = tp.TensorParallelPrefill(config, _tensors(tp.shard_weights(config, weights, lay)), lay,
                                         sequence_length=seq, dtype=np.float32, cache_length=context)
            return list(m.prefill(Tensor(ids), Tensor(selector)))

    ranks = _threaded_ranks(size, build)
    for rank, got in enumerate(ranks):
        lay = tp.shard_layout(config, size, rank)
        np.testing.assert_allclose(got[0], full[0], rtol=0, atol=1e-4 * float(np.abs(full[0]).max()))
        kv = lay.kv_rows.start // config.head_size
        for g, f in zip(got[1:], full[1:]):
            np.testing.assert_allclose(g, f[:, kv:kv + lay.kv_heads], rtol=0, atol=1e-5)


def test_tensor_parallel_plans_lower_the_all_reduce():
    import ml_dtypes

    config, batch, context = TINY, 4, 32
    dt = np.dtype(ml_dtypes.bfloat16)
    weights = {k: v.astype(dt) for k, v in synthetic_weights(config, dtype=np.float32).items()}
    lay = tp.shard_layout(config, 2, 1)
    inputs = _decode_inputs(config, batch, context, 5, seed=1)
    outputs = _tp_decode_graph(config, weights, lay, batch, context, inputs)

    def leaf_dtype(node):
        return np.asarray(node.numpy_value()).dtype

    plan = Planner([o._node for o in outputs], [], backend="cuda-b200", leaf_dtype=leaf_dtype).build()
    reduces = [s for s in plan.steps if s.name == "all_reduce"]
    assert len(reduces) == 2 * config.num_hidden_layers
    assert all(s.args["group"] == "tp" and s.args["src"].dtype == np.float32 for s in reduces)
    assert plan.lowered.get("sdpa") == config.num_hidden_layers
    assert plan.lowered.get("rms_norm") == 2 * config.num_hidden_layers + 1


# ------------------------------------------------------------- gloo ranks
def _gloo_rank(rank: int, size: int, port: int, queue) -> None:
    import os

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        config, batch, context = TINY, 2, 16
        weights = synthetic_weights(config, dtype=np.float32)
        inputs = _decode_inputs(config, batch, context, 4, seed=7)
        outputs = _tp_decode_graph(config, weights, tp.shard_layout(config, size, rank), batch, context, inputs)

        def reduce_fn(x):
            t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32).copy())
            dist.all_reduce(t)
            return t.numpy().astype(x.dtype)

        queue.put((rank, _run(outputs, reduce_fn)[0]))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_decode_over_gloo_processes():
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(queue.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    config, batch, context = TINY, 2, 16
    weights = synthetic_weights(config, dtype=np.float32)
    ids, rotation, attention, write, pos, caches = _decode_inputs(config, batch, context, 4, seed=7)
    with no_grad():
        step = BatchedDecoderStep(config, _tensors(weights), batch=batch, cache_length=context, dtype=np.float32)
        t = [Tensor(v) for v in (ids, rotation, attention, write, pos)]
        ct = [Tensor(c) for c in caches]
        full = _run(step(t[0], t[1], t[2], t[3], list(zip(ct[::2], ct[1::2])), position=t[4]), lambda x: x)
    for rank in range(2):
        np.testing.assert_allclose(got[rank], full[0], rtol=0, atol=1e-4 * float(np.abs(full[0]).max()))
