"""The one-shot peer all-reduce (cb_peer_all_reduce) on two B200s.

Two processes, one GPU each, share their exchange regions over CUDA IPC
(cuda_b200.parallel.init_group with peer=True; the handles travel over a
gloo process group).  Every rank must get the float32 sum of the ranks'
partials in rank order -- bit for bit what NumPy computes -- with and without
the residual add, for ragged and maximal counts, over many calls (the two
buffers alternate) and as replays of a captured CUDA graph.  A second test
makes one rank skip a call: the other rank's bounded wait (shortened to
0.2 s) runs out and reports CB_FLAG_WAIT_PEER, with no GPU fault; both
ranks synchronise before the regions are released.  NVLS stays off (plain
NVLink loads and stores only).  Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

COUNTS = [1, 5, 4096, 65536 + 3, 1 << 20]


def _rank(rank: int, size: int, port: int, queue, mode: str) -> None:
    import os
    import sys

    sys.path[:0] = [os.path.join(os.getcwd(), "chomik-grad_b200"), os.getcwd()]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import numpy as np
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=size)
    result = {}
    try:
        import cuda_b200  # noqa: F401
        from cuda_b200 import _lib, parallel

        comm = parallel.init_group("peer-test", peer=True)
        assert comm.peer
        stream = torch.cuda.current_stream().cuda_stream
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        if mode == "sums":
            bad = []
            for call, count in enumerate(COUNTS * 3):
                parts = [np.random.default_rng(1000 * call + r).normal(0, 1, count).astype(np.float32)
                         for r in range(size)]
                residual = np.random.default_rng(77 + call).normal(0, 1, count).astype(np.float32)
                want = parts[0].copy()
                for p in parts[1:]:
                    want = want + p
                src = torch.from_numpy(parts[rank]).cuda()
                out = torch.full((count,), float("nan"), device="cuda")
                with_res = call % 2 == 1
                res = torch.from_numpy(residual).cuda() if with_res else None
                comm.all_reduce(src.data_ptr(), out.data_ptr(), count, _lib.F32, stream,
                                error_flag=flag.data_ptr(), residual=res.data_ptr() if with_res else None)
                torch.cuda.synchronize()
                expect = residual + want if with_res else want
                if not np.array_equal(out.cpu().numpy(), expect):
                    bad.append((call, count, with_res))
            result["bad"] = bad
            # graph replays: the epoch lives on the device, so one captured launch serves every call
            count = 65536
            src = torch.zeros(count, device="cuda")
            out = torch.zeros(count, device="cuda")
            graph = torch.cuda.CUDAGraph()
            capture = torch.cuda.Stream()
            with torch.cuda.stream(capture):
                with torch.cuda.graph(graph, stream=capture):
                    comm.all_reduce(src.data_ptr(), out.data_ptr(), count, _lib.F32, capture.cuda_stream,
                                    error_flag=flag.data_ptr())
            replay_bad = []
            for i in range(12):
                parts = [np.random.default_rng(5000 + 10 * i + r).normal(0, 1, count).astype(np.float32)
                         for r in range(size)]
                src.copy_(torch.from_numpy(parts[rank]))
                graph.replay()
                torch.cuda.synchronize()
                want = parts[0].copy()
                for p in parts[1:]:
                    want = want + p
                if not np.array_equal(out.cpu().numpy(), want):
                    replay_bad.append(i)
            del graph
            result["replay_bad"] = replay_bad
        else:  # "absent": rank 1 skips the second call
            comm.set_peer_wait(0.2)
            src = torch.ones(4096, device="cuda")
            out = torch.zeros(4096, device="cuda")
            comm.all_reduce(src.data_ptr(), out.data_ptr(), 4096, _lib.F32, stream, error_flag=flag.data_ptr())
            torch.cuda.synchronize()
            result["first_flag"] = int(flag.item())
            result["first_sum"] = float(out[0].item())
            if rank == 0:
                comm.all_reduce(src.data_ptr(), out.data_ptr(), 4096, _lib.F32, stream, error_flag=flag.data_ptr())
                torch.cuda.synchronize()
            result["second_flag"] = int(flag.item())
        result["flag"] = int(flag.item())
        torch.cuda.synchronize()
        dist.barrier()  # every rank's kernels are done before any region is released
        parallel.destroy_group("peer-test")
        queue.put((rank, result))
    except Exception as exc:  # noqa: BLE001
        queue.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def _run(size: int, mode: str) -> dict:
    import multiprocessing as mp
    import queue as queue_mod
    import socket
    import time

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, size, port, queue, mode)) for r in range(size)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 300
    while len(got) < size:
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
    return got


def _two_gpus():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def test_peer_all_reduce_sums_bit_for_bit():
    _two_gpus()
    got = _run(2, "sums")
    for rank, r in got.items():
        assert r["bad"] == [], (rank, r["bad"])
        assert r["replay_bad"] == [], (rank, r["replay_bad"])
        assert r["flag"] == 0, rank


def test_peer_all_reduce_wait_runs_out_when_a_rank_is_absent():
    from cuda_b200 import _lib

    _two_gpus()
    got = _run(2, "absent")
    for rank in range(2):
        assert got[rank]["first_flag"] == 0 and got[rank]["first_sum"] == 2.0
    assert got[0]["second_flag"] == _lib.FLAG_WAIT_PEER
    assert got[1]["second_flag"] == 0
