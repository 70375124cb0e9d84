"""Microbenchmarks of single kernels and of the batched decode step (needs a B200).

    python kernel_bench.py sdpa_tc   [--tokens 2048 --heads 32 --kv 4 --hd 64 --causal 3]
    python kernel_bench.py gemm_tc   [--m 2048 --n 5632 --k 2048]
    python kernel_bench.py sdpa_query [--batch 32 --heads 32 --kv 4 --tokens 768 --hd 64]
    python kernel_bench.py batched   [--workload tinyllama-bf16-bs32 --steps 20 --prompt 64]
    python kernel_bench.py sample    [--rows 1 --width 32000 --top-k 50]
    python kernel_bench.py gemm_rows [--batch 32]

Each prints CUDA-event times (warm, averaged over --reps launches on the
current stream).  ``batched`` wraps the timed graph replays in
cudaProfilerStart/Stop, so ``ncu --profile-from-start off`` sees only them.
Inputs are random; these time kernels, they do not check results (the
``-m gpu`` tests do).
"""

from __future__ import annotations

import argparse
import ctypes
from pathlib import Path
import statistics
import sys

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "baseline" / "_ref", ROOT / "chomik-grad_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402


def _timed(fn, reps: int) -> float:
    import torch

    fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / reps


def _sdpa_args(q, k, v, mask, out, divisor: float):
    import torch

    from cuda_b200 import _lib

    a = _lib.SdpaArgs()
    for name, t in (("q", q), ("k", k), ("v", v), ("mask", mask)):
        setattr(a, name, t.data_ptr())
        setattr(a, f"{name}_dtype", _lib.F32 if t.dtype == torch.float32 else _lib.BF16)
        strides = getattr(a, f"{name}_strides")
        for d in range(4):
            strides[d] = 0 if t.shape[d] == 1 else t.stride(d)
    a.out = out.data_ptr()
    a.batch, a.heads, a.tq, a.head_size = q.shape
    a.kv_heads, a.tk = k.shape[1], k.shape[2]
    a.divisor = divisor
    return a


def sdpa_tc(args) -> None:
    import torch

    from cuda_b200 import _lib

    b, h, kv, t, hd = 1, args.heads, args.kv, args.tokens, args.hd
    q = torch.randn(b, h, t, hd, device="cuda")
    k = torch.randn(b, kv, t, hd, device="cuda")
    v = torch.randn(b, t, kv, hd, device="cuda").permute(0, 2, 1, 3)  # strided, like the model's v
    i, j = torch.arange(t)[:, None], torch.arange(t)[None, :]
    mask = torch.where(j > i, -1e4, 0.0).to(torch.bfloat16).reshape(1, 1, t, t).cuda()
    out = torch.empty(b, h, t, hd, device="cuda")
    a = _sdpa_args(q, k, v, mask, out, float(np.sqrt(hd)))
    lib = _lib.load()
    scratch = torch.empty(lib.cb_sdpa_tc_scratch(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ms = _timed(lambda: _lib.call("cb_sdpa_tc", ctypes.byref(a), args.causal, scratch.data_ptr(),
                                  flag.data_ptr(), stream), args.reps)
    flops = 4.0 * b * h * t * t * hd * (0.5 if args.causal else 1.0)
    print(f"cb_sdpa_tc heads {h}/{kv} tokens {t} hd {hd} causal {args.causal}: {ms * 1000:.1f} us, "
          f"{flops / ms / 1e9:.1f} TFLOP/s of the reference's products, error flag {int(flag.item())}")


def gemm_tc(args) -> None:
    import torch

    from cuda_b200 import _lib

    m, n, k = args.m, args.n, args.k
    a_t = torch.randn(m, k, device="cuda")
    b_t = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    c_t = torch.empty(m, n, device="cuda")
    g = _lib.GemmArgs()
    g.a, g.a_dtype, g.lda = a_t.data_ptr(), _lib.F32, k
    g.b, g.ldb, g.c, g.ldc = b_t.data_ptr(), k, c_t.data_ptr(), n
    g.m, g.n, g.k = m, n, k
    lib = _lib.load()
    scratch = torch.empty(lib.cb_gemm_tc_scratch(ctypes.byref(g)), dtype=torch.uint8, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.a_split, g.error_flag = scratch.data_ptr(), flag.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    ms = _timed(lambda: _lib.call("cb_gemm_tc", ctypes.byref(g), stream), args.reps)
    print(f"cb_gemm_tc float32 A {m}x{k}, W {n}x{k}: {ms * 1000:.1f} us, {2 * m * n * k / ms / 1e9:.0f} TFLOP/s "
          f"of the reference's product, error flag {int(flag.item())}")


def sdpa_query(args) -> None:
    import torch

    from cuda_b200 import _lib

    b, h, kv, t, hd = args.batch, args.heads, args.kv, args.tokens, args.hd
    q = torch.randn(b, h, 1, hd, device="cuda")
    k = torch.randn(b, kv, t, hd, device="cuda")
    v = torch.randn(b, kv, t, hd, device="cuda")
    mask = torch.zeros(1, 1, 1, t, device="cuda")
    out = torch.empty(b, h, 1, hd, device="cuda")
    a = _sdpa_args(q, k, v, mask, out, float(np.sqrt(hd)))
    lib = _lib.load()
    scratch = torch.empty(lib.cb_sdpa_query_scratch(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ms = _timed(lambda: _lib.call("cb_sdpa_query", ctypes.byref(a), scratch.data_ptr(), stream), args.reps)
    print(f"cb_sdpa_query batch {b} heads {h}/{kv} keys {t} hd {hd}: {ms * 1000:.1f} us, "
          f"{2 * b * kv * t * hd * 4 / ms / 1e6:.0f} GB/s of K/V")


def sample(args) -> None:
    import torch

    from cuda_b200 import _lib

    rows, width = args.rows, args.width
    logits = torch.randn(rows, width, device="cuda") * 2.0
    uniforms = torch.rand(rows, dtype=torch.float64, device="cuda")
    out = torch.empty(rows, dtype=torch.int64, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = _lib.SampleArgs()
    a.logits, a.logits_dtype, a.rows, a.width, a.ld = logits.data_ptr(), _lib.F32, rows, width, width
    a.temperature, a.top_k = 0.8, args.top_k
    a.uniforms, a.out, a.error_flag = uniforms.data_ptr(), out.data_ptr(), flag.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    ms = _timed(lambda: _lib.call("cb_sample_rows", ctypes.byref(a), stream), args.reps)
    # what the host sampler needs first: the rows in host memory
    host = torch.empty(rows, width, pin_memory=True)
    copy_ms = _timed(lambda: host.copy_(logits, non_blocking=True), args.reps)
    print(f"cb_sample_rows rows {rows} width {width} top_k {args.top_k}: {ms * 1000:.1f} us "
          f"(device-to-host copy of the rows alone: {copy_ms * 1000:.1f} us), error flag {int(flag.item())}")


def batched(args) -> None:
    import torch

    from cuda_b200.batched import BatchedRuntime
    from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights

    wl = WORKLOADS[args.workload]
    cfg = wl.config
    if cfg.hidden_size >= 4096:  # Llama-3-8B shape: weights drawn on the GPU, the TP = 1 runtime (as bench.py)
        from cuda_b200 import tensor_parallel as tp
        from cuda_b200.models import bfloat16, device_weights

        layout = tp.shard_layout(cfg, 1, 0)
        rt = tp.TensorParallelRuntime(cfg, device_weights(cfg, device=torch.device("cuda", 0), layout=layout), layout,
                                      batch=wl.batch, dtype=bfloat16())
    else:
        rt = BatchedRuntime(cfg, synthetic_weights(cfg, dtype=wl.np_dtype), batch=wl.batch)
    prompts = [list(p) for p in synthetic_prompt(cfg, args.prompt, batch=wl.batch)]
    tokens, caches = rt.prefill_batch(prompts, wl.context)
    rt.decode_batch_on_device(tokens, args.prompt, wl.context, caches, 4)
    torch.cuda.synchronize()
    times: list = []
    torch.cuda.profiler.start()
    rt.decode_batch_on_device(tokens, args.prompt, wl.context, caches, args.steps, replay_times=times)
    torch.cuda.profiler.stop()
    step = statistics.fmean(times)
    print(f"{wl.name}: graph replay {step:.3f} ms per step, {wl.batch / step * 1000:.0f} tokens/s")


ROWS_SHAPES = {  # TinyLlama decode Linears: (weights' row counts, k, x prologue)
    "qkv": ((2048, 256, 256), 2048, "rms"),
    "o": ((2048,), 2048, "plain"),
    "gateup": ((5632, 5632), 2048, "rms"),
    "down": ((2048,), 5632, "swiglu"),
}


def gemm_rows(args) -> None:
    """cb_gemm_rows at the batched decode step's four Linear shapes, one after another.

    Each shape cycles through enough weight copies (> 256 MB) that every launch
    streams its weights from HBM, as the step does; x prologues as in the step
    (RMSNorm before q/k/v and gate/up, SwiGLU before down).  Prints the CUDA-event
    time per launch and the weight bytes over it.
    """
    import torch

    from cuda_b200 import _lib

    lib = _lib.load()
    rows = args.batch
    shapes = {n: s for n, s in ROWS_SHAPES.items() if n in args.shapes}
    for name, (ns, k, mode), splits in ((n, s, c) for n, s in shapes.items() for c in args.splits):
        wbytes = sum(ns) * k * 2
        copies = max(2, -(-256 * 2 ** 20 // wbytes))
        ws = [[(torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16) for n in ns] for _ in range(copies)]
        x = torch.randn(rows, k, device="cuda")
        x2 = torch.randn(rows, k, device="cuda")
        norm_w = torch.ones(k, device="cuda", dtype=torch.bfloat16)
        outs = [torch.empty(rows, n, device="cuda") for n in ns]
        residual = torch.randn(rows, ns[0], device="cuda")
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        launches = []
        for c in range(copies):
            a = _lib.GemmRowsArgs()
            a.x, a.x_dtype, a.ldx = x.data_ptr(), _lib.F32, k
            a.rows, a.k, a.n_w, a.splits, a.pdl = rows, k, len(ns), splits, 1
            for i, (w, o) in enumerate(zip(ws[c], outs)):
                a.w[i], a.w_rows[i], a.out[i], a.ldo[i] = w.data_ptr(), w.shape[0], o.data_ptr(), o.stride(0)
            if mode == "rms":
                a.x_mode, a.norm_w, a.norm_w_dtype = _lib.ROWS_X_RMS, norm_w.data_ptr(), _lib.BF16
                a.divisor, a.eps = float(k), 1e-5
                a.dt_sq = a.dt_sum = a.dt_mean = a.dt_t = a.dt_d = a.dt_y = _lib.F32
                a.dt_out = _lib.BF16
            elif mode == "swiglu":
                a.x_mode, a.x2, a.x2_dtype, a.ldx2 = _lib.ROWS_X_SWIGLU, x2.data_ptr(), _lib.F32, k
            if len(ns) == 1:
                a.residual, a.ldr = residual.data_ptr(), residual.stride(0)
            scratch = torch.empty(max(lib.cb_gemm_rows_scratch(ctypes.byref(a)), 16), dtype=torch.uint8,
                                  device="cuda")
            counters = torch.zeros(max(lib.cb_gemm_rows_counters(ctypes.byref(a)), 1), dtype=torch.int32,
                                   device="cuda")
            a.scratch, a.counters, a.error_flag = scratch.data_ptr(), counters.data_ptr(), flag.data_ptr()
            launches.append((a, scratch, counters))
        it = iter(range(10 ** 9))

        def run():
            _lib.call("cb_gemm_rows", ctypes.byref(launches[next(it) % copies][0]),
                      torch.cuda.current_stream().cuda_stream)

        ms = _timed(run, args.reps)
        # the same launches replayed from a CUDA graph (no host time between them, as in the decode step)
        run()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(copies):
                run()
        graph_ms = _timed(graph.replay, max(1, args.reps // copies)) / copies
        assert int(flag.item()) == 0, f"cb_gemm_rows error flag {int(flag.item())}"
        print(f"gemm_rows {name}: rows {rows} n {ns} k {k} ({mode}) ctas {splits or 'all'}: {ms * 1000:.1f} us per launch from the "
              f"host, {graph_ms * 1000:.1f} us in a graph; {wbytes / 1e6:.1f} MB weights, "
              f"{wbytes / (graph_ms / 1000) / 1e9:.0f} GB/s in the graph")
        del ws, launches, graph
        torch.cuda.empty_cache()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("kernel", choices=("sdpa_tc", "gemm_tc", "sdpa_query", "batched", "sample", "gemm_rows"))
    parser.add_argument("--reps", type=int, default=20)
    parser.add_argument("--splits", type=int, nargs="+", default=[0],
                        help="gemm_rows: CTA counts to time (0: one per SM, the runtime's choice)")
    parser.add_argument("--shapes", nargs="+", default=list(ROWS_SHAPES), choices=list(ROWS_SHAPES),
                        help="gemm_rows: which Linear shapes")
    parser.add_argument("--tokens", type=int, default=None)
    parser.add_argument("--heads", type=int, default=32)
    parser.add_argument("--kv", type=int, default=None)
    parser.add_argument("--hd", type=int, default=64)
    parser.add_argument("--causal", type=int, default=3)
    parser.add_argument("--batch", type=int, default=32)
    parser.add_argument("--m", type=int, default=2048)
    parser.add_argument("--n", type=int, default=5632)
    parser.add_argument("--k", type=int, default=2048)
    parser.add_argument("--workload", default="tinyllama-bf16-bs32")
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--prompt", type=int, default=64)
    parser.add_argument("--rows", type=int, default=1)
    parser.add_argument("--width", type=int, default=32000)
    parser.add_argument("--top-k", type=int, default=50)
    parser.add_argument("--kv-cache", default="bfloat16", choices=("bfloat16", "float32"),
                        help="batched: KV-cache storage (the compiler's kv_cache_dtype), as bench.py")
    args = parser.parse_args()
    import os

    os.environ["CUDA_B200_KV_DTYPE"] = args.kv_cache  # read when the compiler is first created
    if args.kv is None:
        args.kv = 4
    if args.tokens is None:
        args.tokens = 2048 if args.kernel == "sdpa_tc" else 768
    {"sdpa_tc": sdpa_tc, "gemm_tc": gemm_tc, "sdpa_query": sdpa_query, "batched": batched,
     "sample": sample, "gemm_rows": gemm_rows}[args.kernel](args)


if __name__ == "__main__":
    main()
