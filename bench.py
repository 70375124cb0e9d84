"""Decode tokens/s of the cuda-b200 plugin (Llama hot path), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload tinyllama-bf16-bs1]

Workload (default): TinyLlama-1.1B shape, bf16 weights, random init, batch 1,
128-token prompt then greedy decode with a 384-row KV cache (the reference's
``context = prompt + 256`` rule), the cache held in bfloat16 (``--kv-cache
float32`` keeps the reference's float32 cache layout).  A *step* is one decode step (one token).
With N GPUs (torchrun, one process per GPU) every rank decodes its own
sequence: independent replicas, weak scaling, no collective on the data path.

Reported:
  value      device-resident decode: the captured decode graph replayed K
             times with the next step's inputs written on the device from the
             previous argmax (no host round trip), CUDA-event timed, max over
             ranks;  value = N * K / time.
  e2e        the reference's own loop through the public API: per step build
             the host inputs, device.array(...) them, program.run(bindings),
             device.argmax(logits) -- host<->device copies inside the timing.
  roofline   the whole decode step is one persistent kernel (cb_decode_step):
             weight + KV + embedding bytes per launch over its CUDA-event
             time, vs the measured HBM copy bandwidth; step_roofline: the
             same bytes per token x tokens/s.
  prefill    the prefill-heavy config on the same weights: 8 prompts of 2048
             tokens per step (tcgen05 GEMMs and flash attention), tokens/s
             and FLOP/s against the measured bf16 tensor peak.
  bs32       batched decode of 32 sequences (one BatchedDecoderStep program,
             tcgen05 row GEMMs, split-key attention), graph replays; per rank.
  llama3_8b_tp  Llama-3-8B shape, 16 sequences of 1024-token prompts, prefill
             then batched decode, tensor-parallel over all N ranks (TP = N,
             NCCL all-reduce inside each rank's decode graph); tokens/s of the
             group and the fraction of the group's aggregate HBM bandwidth.
  cpu_baseline  the unmodified reference's own cpu compiler (from baseline/_ref)
             timing real decode steps of the same model on the host cores:
             the float32 model on the bf16-rounded weights (BLAS threads
             measured), and beside it the bf16 model as the reference's loop
             runs it (cpu_baseline_bf16_literal).
Inputs are larger than L2 (2.07 GB of weights per step), so no flush is needed.
"""

from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import statistics
import subprocess
import sys
import threading
import time

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "baseline" / "_ref", ROOT / "chomik-grad_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402

METRIC = ("decode tokens/sec (bs=1; bs=32 in the bs32 object; Llama-3-8B bs16 tensor-parallel in "
          "llama3_8b_tp) and % of HBM roofline")
# DRAM bytes of one gate/up GEMV launch from an ncu capture, per workload
GATEUP_TRAFFIC = {"tinyllama-bf16-bs1": 56_449_792 + 45_312}
# DRAM bytes of one cb_decode_step launch from an ncu capture, per (workload, KV-cache dtype)
STEP_TRAFFIC = {("tinyllama-bf16-bs1", "float32"): 2_091_113_000 + 7_491_584,
                ("tinyllama-bf16-bs1", "bfloat16"): 2_082_805_000 + 8_020_736}
PEAKS = ROOT / "MEASURED_PEAKS.json"


def measured_peaks():
    try:
        data = json.loads(PEAKS.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a while to start: the timed region begins after its first
            # sample, so a short region still gets samples (bounded: 5 s)
            deadline = time.time() + 5.0
            while not self.lines and self.proc.poll() is None and time.time() < deadline:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def dist_setup(gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def reduce_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def weight_bytes(config, itemsize: int) -> int:
    from chomikgrad.llama import required_weight_shapes

    total = sum(int(np.prod(s)) for n, s in required_weight_shapes(config).items()
                if n != "model.embed_tokens.weight")
    return total * itemsize


def kv_name() -> str:
    """The KV-cache storage the b200 compiler was created with (the CUDA_B200_KV_DTYPE it read)."""
    return os.environ.get("CUDA_B200_KV_DTYPE", "float32")


def kv_itemsize() -> int:
    return 2 if kv_name() == "bfloat16" else 4


def blas_threads() -> int:
    """Threads NumPy's BLAS uses (threadpoolctl), after a first matmul loaded it."""
    import threadpoolctl

    np.ones((64, 64), np.float32) @ np.ones((64, 64), np.float32)
    counts = [info.get("num_threads", 1) for info in threadpoolctl.threadpool_info() if info.get("user_api") == "blas"]
    return max(counts) if counts else 1


def cpu_baseline(wl, weights, budget_s: float = 25.0, mode: str = "fp32"):
    """Decode steps of the same model on the host cores through the UNMODIFIED reference's own
    ``cpu`` compiler (chomikgrad.lazy.NumpyCompiler, imported from baseline/_ref), in a bounded sample.

    mode "fp32": the model in float32 on the bf16-rounded weights -- every matmul a float32 BLAS
    call on all the BLAS threads (the fastest the reference runs this model on a CPU);
    mode "bf16": the bf16 model as the reference's loop runs it, whose first matmul per layer
    runs in ml_dtypes bfloat16 loops (single-threaded) and the rest in float32.
    """
    import chomikgrad

    from cuda_b200.runtime import LlamaRuntime

    assert type(chomikgrad.get_compiler("cpu")).__module__ == "chomikgrad.lazy", "cpu must be the reference's"
    cfg = wl.config
    dtype = np.dtype(np.float32) if mode == "fp32" else wl.np_dtype
    host = {k: np.asarray(v).astype(dtype) for k, v in weights.items()} if mode == "fp32" else weights
    rt = LlamaRuntime(cfg, host, compiler="cpu", dtype=dtype)
    context = wl.context
    shape = (1, cfg.num_key_value_heads, context, cfg.head_size)
    caches = [np.zeros(shape, np.float32) for _ in range(2 * cfg.num_hidden_layers)]
    position = wl.prompt_tokens
    times = []
    started = time.perf_counter()
    token = 1
    while True:
        t0 = time.perf_counter()
        logits, caches = rt.decode(token, position, context, caches)
        token = rt.device.argmax(logits)
        times.append(time.perf_counter() - t0)
        position += 1
        if position >= context:  # keep inside the cache (small configs reach it within the sample)
            position = wl.prompt_tokens
        if time.perf_counter() - started > budget_s or len(times) >= 50:
            break
    warm = times[1:] if len(times) > 1 else times
    per_token = statistics.median(warm)
    threads = blas_threads() if mode == "fp32" else 1
    what = ("float32 model on the bf16-rounded weights, every matmul a float32 BLAS call" if mode == "fp32" else
            "bf16 model as the reference's loop runs it (first matmul per layer in single-threaded ml_dtypes "
            "bfloat16 loops, the rest float32)")
    return {"value": 1.0 / per_token, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{len(times)} decode steps (first excluded if >1) of {wl.name} at context {context} through "
                      f"the unmodified reference's cpu compiler (chomikgrad.lazy.NumpyCompiler): {what}; "
                      f"NumPy {np.__version__}, {threads} BLAS thread(s) used, {os.cpu_count()} host cores",
            "seconds_per_token": per_token, "mode": mode}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from cuda_b200.models import WORKLOADS, synthetic_weights

    wl = WORKLOADS[args.workload]
    weights = synthetic_weights(wl.config, dtype=wl.np_dtype)
    budget = float(os.environ.get("CB_REFERENCE_BUDGET_S", "150"))
    base = cpu_baseline(wl, weights, budget_s=budget, mode=args.reference_mode)
    line = {
        "metric": METRIC, "value": base["value"], "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * base["seconds_per_token"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if args.reference_mode == "fp32" else "bf16",
        "data": "synthetic",
        "config": {"workload": wl.name, "model": "TinyLlama-1.1B-shape (random init)", "global_batch": 1,
                   "prompt_tokens": wl.prompt_tokens, "context": wl.context,
                   "reference_mode": args.reference_mode},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemv_roofline(program, rounds: int = 20):
    """Average duration of the fused gate/up GEMV, all layers' weights in turn."""
    import torch

    from cuda_b200 import _lib

    steps = [s for s in program.plan.steps if s.name == "gemv" and s.args["epilogue"] == _lib.EPI_SILU_MUL]
    stream = program.device.stream()
    for s in steps:
        program._step_gemv(s, stream)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(rounds):
        for s in steps:
            program._step_gemv(s, stream)
    end.record()
    end.synchronize()
    per_launch_ms = start.elapsed_time(end) / (rounds * len(steps))
    nbytes = sum(v.buf.size * v.dtype.itemsize for v in steps[0].args["weights"])
    return nbytes, per_launch_ms, len(steps)


def prefill_flops(cfg, tokens: int) -> float:
    """FLOPs of one prompt: 2 x non-embedding, non-lm_head parameters x tokens,
    causal attention L x 2 x T^2 x H, and the lm_head row (2 x V x H)."""
    h, kv = cfg.hidden_size, cfg.num_key_value_heads * cfg.head_size
    body = cfg.num_hidden_layers * (h * (h + 2 * kv) + h * h + 3 * h * cfg.intermediate_size)
    return (2.0 * body * tokens + cfg.num_hidden_layers * 2.0 * tokens * tokens * h
            + 2.0 * cfg.vocab_size * h)


def prefill_measurement(rt, cfg, rank: int, world: int, steps: int, warmup: int) -> dict:
    """Prefill-heavy config: 8 prompts of 2048 tokens per step, one greedy token each.

    The 8 prompts run as one program (``LlamaRuntime.prefill_batched``: the
    reference's prefill graph with its batch dimension, every Linear one GEMM
    over all 16384 rows); the output tokens are the argmax of each prompt's
    logits row.  Timed with CUDA events on the launching stream, max over ranks.
    """
    import torch

    from cuda_b200.models import WORKLOADS, synthetic_prompt

    wl = WORKLOADS["tinyllama-bf16-prefill-bs8"]
    prompts = [list(p) for p in synthetic_prompt(cfg, wl.prompt_tokens, seed=100 + rank, batch=wl.batch)]
    context = wl.prompt_tokens

    def one_step():
        return rt.prefill_batched(prompts, context)[0]

    for _ in range(max(warmup, 1)):
        one_step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        logits = one_step()
    t1.record()
    t1.synchronize()
    ms = reduce_max(t0.elapsed_time(t1), world)
    tokens = wl.batch * wl.prompt_tokens * steps * world
    first_tokens = [int(t) for t in rt.device.argmax_last_axis(logits)]
    flops = prefill_flops(cfg, wl.prompt_tokens) * wl.batch * steps * world
    # the group's peak: every rank prefills its own prompts (replicas), so the
    # whole job's FLOP/s is measured against world x one B200's peak
    peak = (json.loads(PEAKS.read_text())["bf16_tflops"] if PEAKS.exists() else 1590.0) * world
    achieved = flops / (ms / 1000.0) / 1e12
    program = rt._prefill[("batched", wl.batch, wl.prompt_tokens, context)][0]
    return {"workload": wl.name, "value": tokens / (ms / 1000.0), "unit": "tokens/s",
            "ms_per_step": ms / steps, "steps": steps, "sequences_per_step": wl.batch * world,
            "first_tokens": first_tokens,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "flops_per_sequence": prefill_flops(cfg, wl.prompt_tokens),
                         "peak_source": "measured" if PEAKS.exists() else "fallback"},
            "gpu_launches": program.launches * steps}


def rows_roofline(rt, rows: int, rounds: int = 3):
    """The gate/up cb_gemm_rows launch (largest weight stream of a batched step) timed
    alone with CUDA events, cycling every layer's weights (> L2): algorithmic bytes
    (both weights + x + out) per launch over the mean launch time."""
    import ctypes

    import torch

    from cuda_b200 import _lib

    cfg = rt.config
    dev = rt.device.torch_device
    x = torch.randn(rows, cfg.hidden_size, device=dev)
    outs = [torch.empty(rows, cfg.intermediate_size, device=dev) for _ in range(2)]
    lib = _lib.load()
    args = []
    for layer in range(cfg.num_hidden_layers):
        g = _lib.GemmRowsArgs()
        g.x, g.x_dtype, g.ldx, g.rows, g.k, g.n_w = x.data_ptr(), _lib.F32, cfg.hidden_size, rows, cfg.hidden_size, 2
        for i, name in enumerate(("gate_proj", "up_proj")):
            w = rt.weights[f"model.layers.{layer}.mlp.{name}.weight"]
            g.w[i] = rt.device.array(w._node.native_values[rt.device.name]).data_ptr()
            g.w_rows[i], g.out[i], g.ldo[i] = cfg.intermediate_size, outs[i].data_ptr(), cfg.intermediate_size
        args.append(g)
    scratch = torch.empty(lib.cb_gemm_rows_scratch(ctypes.byref(args[0])), dtype=torch.uint8, device=dev)
    counters = torch.zeros(lib.cb_gemm_rows_counters(ctypes.byref(args[0])), dtype=torch.int32, device=dev)
    for g in args:
        g.scratch, g.counters = scratch.data_ptr(), counters.data_ptr()
    stream = rt.device.stream()
    for g in args:
        _lib.call("cb_gemm_rows", ctypes.byref(g), stream)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(rounds):
        for g in args:
            _lib.call("cb_gemm_rows", ctypes.byref(g), stream)
    t1.record()
    t1.synchronize()
    ms = t0.elapsed_time(t1) / (rounds * len(args))
    nbytes = 2 * cfg.intermediate_size * cfg.hidden_size * 2 + rows * cfg.hidden_size * 4 \
        + 2 * rows * cfg.intermediate_size * 4
    return nbytes, ms


def batched_measurement(cfg, weights, rank: int, world: int, steps: int, warmup: int) -> dict:
    """Batched decode: 32 sequences of 512-token prompts stepped together (one
    BatchedDecoderStep program), each step one token of every sequence."""
    import torch

    from cuda_b200.batched import BatchedRuntime
    from cuda_b200.models import WORKLOADS, synthetic_prompt

    wl = WORKLOADS["tinyllama-bf16-bs32"]
    rt = BatchedRuntime(cfg, weights, batch=wl.batch, compiler="cuda-b200")
    prompts = [list(p) for p in synthetic_prompt(cfg, wl.prompt_tokens, seed=200 + rank, batch=wl.batch)]
    context = wl.context
    start = wl.prompt_tokens
    tokens, caches = rt.prefill_batch(prompts, context)
    per_chunk = context - start - 2
    rt.decode_batch_on_device(tokens, start, context, caches, min(max(warmup, 3), per_chunk))
    barrier(world)
    replay_ms: list = []
    elapsed, done = 0.0, 0
    while done < steps:
        n = min(per_chunk, steps - done)
        _, ms = rt.decode_batch_on_device(tokens, start, context, caches, n + 1, replay_times=replay_ms)
        elapsed += ms
        done += n
    slowest = reduce_max(elapsed, world)
    value = steps * wl.batch * world / (slowest / 1000.0)

    # e2e: host loop through the public API (inputs uploaded, argmax read back every step)
    def host_steps(n: int):
        nonlocal caches
        toks, position = list(tokens), start
        for _ in range(n):
            logits, caches = rt.decode_batch(toks, position, context, caches)
            toks = [int(t) for t in rt.device.argmax_last_axis(logits)]
            position += 1
    e2e_steps = min(steps, per_chunk)
    host_steps(2)
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    host_steps(e2e_steps)
    t1.record()
    t1.synchronize()
    e2e_ms = reduce_max(t0.elapsed_time(t1), world)
    host = rt.batched_step_inputs(tokens, start, context)
    program = next(iter(rt._batched.values()))[0]

    peak, peak_kind = measured_peaks()
    kv_read = wl.batch * 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_size * kv_itemsize() * context
    step_bytes = weight_bytes(cfg, 2) + wl.batch * cfg.hidden_size * 2 + kv_read
    step_ms = statistics.fmean(replay_ms)
    rbytes, rms = rows_roofline(rt, wl.batch)
    return {
        "workload": wl.name, "value": value, "unit": "tokens/s", "sequences": wl.batch * world,
        "kv_cache": kv_name(),
        "steps": steps, "ms_per_step": slowest / steps,
        "e2e": {"value": e2e_steps * wl.batch * world / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": int(sum(a.nbytes for a in host)), "d2h_bytes_per_step": 8 * wl.batch},
        "roofline": {"bound": "hbm", "achieved": rbytes / (rms / 1000.0) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": rbytes / (rms / 1000.0) / 1e9 / peak, "traffic": None,
                     "kernel": f"cb_gemm_rows gate/up ({rbytes / 1e6:.1f} MB per launch, "
                               f"{cfg.num_hidden_layers} layers cycled)", "kernel_ms": rms,
                     "peak_source": peak_kind},
        "step_roofline": {"bytes_per_step": step_bytes, "achieved": step_bytes / (step_ms / 1000.0) / 1e9,
                          "peak": peak, "unit": "GB/s",
                          "frac": step_bytes / (step_ms / 1000.0) / 1e9 / peak,
                          "basis": f"bf16 weights + {kv_name()} K/V over the whole context (the attention "
                                   "reads every cache row) per step of 32 tokens"},
        "gpu_launches": (program.launches + 2) * steps,
    }


def llama3_measurement(rank: int, world: int, local: int, steps: int, warmup: int, prompt_len: int,
                       vocab_shard: bool = False) -> dict:
    """Llama-3-8B shape, batch 16, tensor-parallel over all ranks (TP = world size).

    Weights are random-init bf16 drawn on each GPU (cuda_b200.models.device_weights)
    and sharded by cuda_b200.tensor_parallel; the all-reduce after the O and
    down projections is an NCCL step inside each rank's captured decode graph.
    Tokens per step are the 16 sequences (shared by every rank).
    """
    import torch

    from cuda_b200 import parallel, tensor_parallel as tp
    from cuda_b200.models import WORKLOADS, bfloat16, device_weights, synthetic_prompt
    from chomikgrad.llama import required_weight_shapes

    wl = WORKLOADS["llama3-8b-bf16-bs16"]
    cfg = wl.config
    if world > 1:
        parallel.init_group("tp")
    layout = tp.shard_layout(cfg, world, rank, vocab_shard=vocab_shard)
    weights = device_weights(cfg, device=torch.device("cuda", local), layout=layout)
    rt = tp.TensorParallelRuntime(cfg, weights, layout, batch=wl.batch, dtype=bfloat16())
    context = prompt_len + wl.decode_steps
    prompts = [list(p) for p in synthetic_prompt(cfg, prompt_len, seed=300, batch=wl.batch)]
    # one whole untimed batch first: compiles the batched prefill program and allocates its buffers
    tokens, caches = rt.prefill_batch(prompts, context)
    del caches
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    tokens, caches = rt.prefill_batch(prompts, context)
    t1.record()
    t1.synchronize()
    prefill_ms = reduce_max(t0.elapsed_time(t1), world)
    rt.decode_batch_on_device(tokens, prompt_len, context, caches, max(warmup, 3))
    barrier(world)
    replay_ms: list = []
    per_chunk = context - prompt_len - 2
    elapsed, done = 0.0, 0
    while done < steps:
        n = min(per_chunk, steps - done)
        _, ms = rt.decode_batch_on_device(tokens, prompt_len, context, caches, n + 1, replay_times=replay_ms)
        elapsed += ms
        done += n
    slowest = reduce_max(elapsed, world)
    step_ms = reduce_max(statistics.fmean(replay_ms), world)
    rt.close()  # release the graphs that hold NCCL work before the communicator
    nccl = None
    if world > 1:
        allreduce = "peer one-shot (NVLink stores, CUDA IPC)" if parallel.get_group("tp").peer else "nccl"
        barrier(world)
        parallel.destroy_group("tp")
        del rt, caches
        torch.cuda.empty_cache()
        # the same decode with every all-reduce on NCCL, for comparison (fewer steps)
        parallel.init_group("tp-nccl", peer=False)
        rt2 = tp.TensorParallelRuntime(cfg, weights, layout, batch=wl.batch, dtype=bfloat16(), group="tp-nccl")
        tokens2, caches2 = rt2.prefill_batch(prompts, context)
        rt2.decode_batch_on_device(tokens2, prompt_len, context, caches2, max(warmup, 3))
        barrier(world)
        nccl_times: list = []
        rt2.decode_batch_on_device(tokens2, prompt_len, context, caches2, min(steps, per_chunk) + 1,
                                   replay_times=nccl_times)
        nccl_ms = reduce_max(statistics.fmean(nccl_times), world)
        rt2.close()
        barrier(world)
        parallel.destroy_group("tp-nccl")
        nccl = {"allreduce": "nccl", "ms_per_step": nccl_ms, "value": wl.batch / (nccl_ms / 1000.0),
                "unit": "tokens/s", "steps": min(steps, per_chunk)}
    else:
        allreduce = "none (one rank)"
    peak, peak_kind = measured_peaks()
    flops = json.loads(PEAKS.read_text())["bf16_tflops"] if PEAKS.exists() else 1590.0
    weight_bytes_model = sum(int(np.prod(s)) for n, s in required_weight_shapes(cfg).items()
                             if n != "model.embed_tokens.weight") * 2
    kv_bytes = wl.batch * 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_size * kv_itemsize() * context
    step_bytes = weight_bytes_model + kv_bytes
    achieved = step_bytes / (step_ms / 1000.0) / 1e9
    pflops = prefill_flops(cfg, prompt_len) * wl.batch / (prefill_ms / 1000.0) / 1e12
    return {
        "workload": wl.name, "tensor_parallel": world, "sequences": wl.batch, "prompt_tokens": prompt_len,
        "kv_cache": kv_name(),
        "lm_head": "vocab-sharded, distributed argmax" if vocab_shard else "replicated",
        "allreduce": allreduce,
        "context": context, "value": steps * wl.batch / (slowest / 1000.0), "unit": "tokens/s",
        "ms_per_step": step_ms,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
                     "frac": achieved / (peak * world), "bytes_per_step": step_bytes,
                     "basis": f"bf16 weights (embedding excluded, lm_head once) + {kv_name()} K/V over the context, "
                              "per step of 16 tokens, against the aggregate HBM bandwidth of the group",
                     "peak_source": peak_kind},
        "prefill": {"value": wl.batch * prompt_len / (prefill_ms / 1000.0), "unit": "tokens/s",
                    "ms": prefill_ms, "tflops": pflops, "frac_of_bf16_peak": pflops / (flops * world)},
        "data": "random-init bf16 weights drawn on the GPU (seeded), uniform random prompt ids",
        "decode_nccl_allreduce": nccl,
    }


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", default="b200", choices=("b200", "reference"))
    parser.add_argument("--workload", default="tinyllama-bf16-bs1")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--reference-mode", default="fp32", choices=("fp32", "bf16"),
                        help="--impl reference: the reference cpu compiler on the float32 model (bf16-rounded "
                             "weights, BLAS on every core; the default) or on the bf16 model as its loop runs it")
    parser.add_argument("--bs32-steps", type=int, default=100,
                        help="batched decode steps (32 sequences each) of the bs32 measurement; 0 skips it")
    parser.add_argument("--prefill-steps", type=int, default=2,
                        help="steps (8 prompts of 2048 tokens each) of the prefill measurement; 0 skips it")
    parser.add_argument("--llama3-steps", type=int, default=30,
                        help="tensor-parallel Llama-3-8B bs16 decode steps (TP = GPUs); 0 skips it")
    parser.add_argument("--llama3-prompt", type=int, default=1024, help="Llama-3-8B prompt tokens")
    parser.add_argument("--kv-cache", default="bfloat16", choices=("bfloat16", "float32"),
                        help="KV-cache storage of every b200 measurement (the compiler's kv_cache_dtype)")
    parser.add_argument("--lm-head", default="auto", choices=("auto", "replicated", "vocab-shard"),
                        help="Llama-3-8B: the lm_head's rows replicated, or sharded over the ranks with a distributed "
                             "argmax (auto: sharded when TP > 1)")
    args = parser.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch

    os.environ["CUDA_B200_KV_DTYPE"] = args.kv_cache  # read when the compiler is first created
    rank, world, local = dist_setup(args.gpus)
    import cuda_b200  # noqa: F401
    from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights
    from cuda_b200.runtime import LlamaRuntime

    wl = WORKLOADS[args.workload]
    cfg = wl.config
    weights = synthetic_weights(cfg, dtype=wl.np_dtype)
    rt = LlamaRuntime(cfg, weights, compiler="cuda-b200")
    prompt = list(synthetic_prompt(cfg, wl.prompt_tokens, seed=rank)[0])
    context = wl.context
    start_pos = len(prompt)
    per_chunk = context - start_pos - 2  # decode steps available per pass over the cache

    logits, caches = rt.prefill(prompt, context)
    first = rt.device.argmax(logits)
    program, nodes = rt.decode_program(context, caches, first, start_pos)

    # ---- value: device-resident decode (graph replays, device-side inputs) ----
    replay_ms = []  # device time of each replayed step (CUDA events on the launching stream)

    def device_pass(n_steps: int, times=None):
        return rt.decode_on_device(first, start_pos, context, caches, n_steps + 1, timed=True,
                                   replay_times=times)

    device_pass(min(args.warmup, per_chunk))
    barrier(world)
    elapsed_ms, done = 0.0, 0
    with ClockSampler(local) as clocks:
        while done < args.steps:
            n = min(per_chunk, args.steps - done)
            _, ms = device_pass(n, replay_ms)
            elapsed_ms += ms
            done += n
    barrier(world)
    slowest = reduce_max(elapsed_ms, world)
    tokens_total = args.steps * world
    value = tokens_total / (slowest / 1000.0)

    # ---- e2e: the reference's host loop through the public API ----
    def host_steps(n: int):
        nonlocal caches
        token, position = first, start_pos
        for _ in range(n):
            out, caches = rt.decode(token, position, context, caches)
            token = rt.device.argmax(out)
            position += 1
            if position >= context - 1:
                token, position = first, start_pos

    host_steps(args.warmup)
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    host_steps(args.steps)
    t1.record()
    t1.synchronize()
    e2e_ms = reduce_max(t0.elapsed_time(t1), world)
    e2e_value = tokens_total / (e2e_ms / 1000.0)
    host = rt.step_inputs(first, start_pos, context)
    h2d = int(sum(a.nbytes for a in host))
    d2h = 16

    # ---- roofline of the dominant kernel and of the whole step ----
    peak, peak_kind = measured_peaks()
    itemsize = wl.np_dtype.itemsize
    avg_ctx = start_pos + min(args.steps, per_chunk) / 2
    kv_item = kv_itemsize()
    kv_bytes = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_size * kv_item * context
    step_bytes = weight_bytes(cfg, itemsize) + cfg.hidden_size * itemsize + kv_bytes
    step_gbs = step_bytes * (value / world) / 1e9
    if program.step_mode:
        # the whole step is one cb_decode_step launch: its bytes over its own time
        kernel_ms = statistics.fmean(replay_ms)
        achieved = step_bytes / (kernel_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": STEP_TRAFFIC.get((wl.name, args.kv_cache)),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                      "decode-step launch (profiles/decode_step_tinyllama_bf16_bs1.txt)",
                    "kernel": f"cb_decode_step (whole decode step, {step_bytes / 1e9:.3f} GB per launch: "
                              f"weights + {args.kv_cache} K/V over the {context}-row cache (the attention "
                              f"reads every row, masked ones included) + embedding row)",
                    "kernel_ms": kernel_ms, "peak_source": peak_kind}
    else:
        gemv_bytes, gemv_ms, gemv_layers = gemv_roofline(program)
        achieved = gemv_bytes / (gemv_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": GATEUP_TRAFFIC.get(wl.name),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one gate/up "
                                      "launch (profiles/gemv_per_kernel_tinyllama_bf16_bs1.txt; cold cache, "
                                      "includes its L2 prefetch of the next launch's weights)",
                    "kernel": f"cb_gemv silu_mul (gate/up {gemv_bytes / 1e6:.1f} MB per launch, "
                              f"{gemv_layers} layers cycled)", "peak_source": peak_kind}

    launches_per_step = program.launches + 1  # + cb_decode_advance
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": slowest / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02), uniform random prompt ids)",
        "config": {"workload": wl.name, "model": "TinyLlama-1.1B-shape", "global_batch": world,
                   "seq_len": context, "prompt_tokens": wl.prompt_tokens, "kv_cache": args.kv_cache,
                   "parallelism": f"replicas x{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (2.07 GB weights per step)"},
        "roofline": roofline,
        "step_roofline": {"bytes_per_token": step_bytes, "achieved": step_gbs, "peak": peak,
                          "unit": "GB/s", "frac": step_gbs / peak, "avg_context": avg_ctx},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if args.bs32_steps > 0 and WORKLOADS["tinyllama-bf16-bs32"].config == cfg:
        line["bs32"] = batched_measurement(cfg, weights, rank, world, args.bs32_steps, args.warmup)
    if args.prefill_steps > 0 and WORKLOADS["tinyllama-bf16-prefill-bs8"].config == cfg:
        line["prefill"] = prefill_measurement(rt, cfg, rank, world, args.prefill_steps, 1)
    if args.llama3_steps > 0 and args.workload == "tinyllama-bf16-bs1":
        line["llama3_8b_tp"] = llama3_measurement(rank, world, local, args.llama3_steps, args.warmup,
                                                  args.llama3_prompt,
                                                  args.lm_head == "vocab-shard" or (args.lm_head == "auto" and world > 1))
    if rank == 0 and not args.no_cpu_baseline:
        keys = ("value", "unit", "cores", "kind", "sample")
        line["cpu_baseline"] = {k: v for k, v in cpu_baseline(wl, weights, mode="fp32").items() if k in keys}
        line["cpu_baseline_bf16_literal"] = {k: v for k, v in cpu_baseline(wl, weights, budget_s=15.0,
                                                                           mode="bf16").items() if k in keys}
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
