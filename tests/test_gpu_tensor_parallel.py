"""Tensor-parallel decode on two B200s against the one-GPU plugin.

Two processes, one per GPU, run cuda_b200.tensor_parallel's prefill and
batched decode over their shards; the all-reduce after the O and down
projections is an NCCL step of each compiled program (cuda_b200.parallel),
replayed inside the decode step's CUDA graph.  Every rank must produce the
one-GPU program's greedy tokens, and logits equal up to the float32
reassociation of the sharded sums.  Skipped on a machine with fewer than two
GPUs.  With a vocabulary-sharded lm_head each rank's decode step returns its
columns of the logits and the greedy tokens come from the distributed argmax
(cb_argmax_rows_sharded: records all-gathered by NCCL, inside the captured
graph for the replays); ``full_logits`` gathers whole rows for the logit
check.  On one GPU, a one-rank group with a vocabulary-sharded lm_head runs
the same checks.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _rank(rank: int, size: int, port: int, queue, vocab_shard: bool = False) -> None:
    import os
    import sys

    sys.path[:0] = [os.path.join(os.getcwd(), "chomik-grad_b200"), os.getcwd()]
    import numpy as np
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        import cuda_b200  # noqa: F401
        from cuda_b200 import parallel, tensor_parallel as tp
        from cuda_b200.batched import BatchedRuntime
        from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights

        parallel.init_group("tp")
        wl = WORKLOADS["tiny-bf16"]
        cfg, batch, prompt_len, steps = wl.config, 4, 16, 10
        weights = synthetic_weights(cfg, dtype=wl.np_dtype)
        layout = tp.shard_layout(cfg, size, rank, vocab_shard=vocab_shard)
        rt = tp.TensorParallelRuntime(cfg, tp.shard_weights(cfg, weights, layout), layout, batch=batch)
        prompts = [list(p) for p in synthetic_prompt(cfg, prompt_len, batch=batch)]
        context = prompt_len + steps + 2
        first, caches = rt.prefill_batch(prompts, context)
        host = [list(first)]
        tokens, logits = first, None
        for i in range(steps):
            logits, caches = rt.decode_batch(tokens, prompt_len + i, context, caches)
            tokens = rt.greedy_rows(logits)
            host.append(tokens)
        result = {"host": host, "logits": rt.device.to_numpy(rt.full_logits(logits)).astype(np.float32)}
        # the same steps again as graph replays (NCCL inside the captured graph)
        first2, caches2 = rt.prefill_batch(prompts, context)
        replayed, _ = rt.decode_batch_on_device(first2, prompt_len, context, caches2, steps + 1)
        result["replayed"] = replayed
        if rank == 0:
            one = BatchedRuntime(cfg, weights, batch=batch)
            f1, c1 = one.prefill_batch(prompts, context)
            ref, toks, lg = [list(f1)], f1, None
            for i in range(steps):
                lg, c1 = one.decode_batch(toks, prompt_len + i, context, c1)
                toks = [int(t) for t in one.device.argmax_last_axis(lg)]
                ref.append(toks)
            result["one_gpu"] = ref
            result["one_gpu_logits"] = one.device.to_numpy(lg).astype(np.float32)
        queue.put((rank, result))
        rt.close()  # the graphs hold NCCL work of the group: release them before the communicator
        dist.barrier()
        parallel.destroy_group("tp")
    except Exception as exc:  # noqa: BLE001
        queue.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def _run_group(size: int, vocab_shard: bool) -> None:
    import multiprocessing as mp
    import socket

    import numpy as np

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, size, port, queue, vocab_shard)) for r in range(size)]
    for p in procs:
        p.start()
    got = {}
    import queue as queue_mod
    import time

    deadline = time.time() + 300
    while len(got) < len(procs):  # fail fast if a rank died without reporting
        try:
            rank, result = queue.get(timeout=5)
            got[rank] = result
        except queue_mod.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead and time.time() < deadline, f"rank processes failed: {dead}"
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for rank in range(size):
        assert isinstance(got[rank], dict), got[rank]
    ref = got[0]["one_gpu"]
    scale = float(np.abs(got[0]["one_gpu_logits"]).max())
    for rank in range(size):
        r = got[rank]
        assert r["host"] == ref, (rank, r["host"], ref)
        np.testing.assert_allclose(r["logits"], got[0]["one_gpu_logits"], rtol=0, atol=1e-3 * scale)
        # graph replays: entry i of sequence b is the token decoded at step i (after the prefill's)
        assert [list(col) for col in zip(*r["replayed"])][: len(ref) - 1] == ref[1:], rank


@pytest.mark.parametrize("vocab_shard", [False, True])
def test_tensor_parallel_decode_on_two_gpus_matches_one_gpu(vocab_shard):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_group(2, vocab_shard)


def test_one_rank_group_with_a_sharded_lm_head_matches_one_gpu():
    pytest.importorskip("torch")
    _run_group(1, True)
