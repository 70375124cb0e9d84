"""Generate the golden fixtures in this directory from the REAL reference.

Run in a container where the reference package is importable (its checkout
path is passed with --reference); the GPU test machines never run this file,
they only read the ``.npz`` fixtures it writes:

    python tests/golden/make_golden.py --reference <path-to-chomik-grad> [case ...]

Every fixture comes from the reference's own ``cpu`` compiler executing the
reference's own graphs (``chomikgrad.llama`` builders, ``compile_graph``,
``CompiledProgram.run`` and ``DeviceAdapter.argmax``), driven the way
``examples/generate_tinyllama.py:_generate_loaded`` (:678-857) drives them with
temperature 0, except that generation does not stop at EOS (random weights).
Weights and prompts come from ``cuda_b200.models`` (seeded, see there).
"""

from __future__ import annotations

import argparse
from pathlib import Path
import sys
import time

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "chomik-grad_b200"))
sys.dont_write_bytecode = True


def _reference(path: str):
    sys.path.insert(0, path)
    sys.path.insert(0, str(Path(path) / "examples"))
    import chomikgrad  # noqa: F401
    from chomikgrad import Tensor, compile_graph, get_compiler, no_grad
    from chomikgrad import llama as L

    return Tensor, compile_graph, get_compiler, no_grad, L


def six_ops(ref) -> dict:
    """Known answers for the generic six-op lowering (patterns of test_cuda.py:32-126)."""
    Tensor, compile_graph, get_compiler, no_grad, L = ref
    rng = np.random.default_rng(19)
    out = {}
    left = np.array([[1.0, -2.0, 0.5], [3.0, 4.0, -1.0]], dtype=np.float32)
    right = np.array([[2.0, 1.0], [-1.0, 0.5], [3.0, -2.0]], dtype=np.float32)
    r = (((Tensor(left) @ Tensor(right)).relu() + 0.25).permute(1, 0).reshape(1, 4).sum(axis=1))
    out["chain_left"], out["chain_right"], out["chain_out"] = left, right, r.numpy(compiler="cpu")
    table = np.array([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]], dtype=np.float32)
    idx = np.array([[2, 0, 2]], dtype=np.int32)
    out["gather_table"], out["gather_idx"] = table, idx
    out["gather_out"] = Tensor(table).gather(Tensor(idx, copy=False)).numpy(compiler="cpu")
    a = rng.normal(size=(2, 4, 3, 5)).astype(np.float32)
    b = rng.normal(size=(2, 4, 5, 6)).astype(np.float32)
    out["bmm_a"], out["bmm_b"] = a, b
    out["bmm_out"] = (Tensor(a) @ Tensor(b)).numpy(compiler="cpu")
    p = rng.normal(size=(2, 4, 5)).astype(np.float32)
    w = rng.normal(size=(5, 7)).astype(np.float32)
    out["proj_x"], out["proj_w"] = p, w
    out["proj_out"] = (Tensor(p) @ Tensor(w)).numpy(compiler="cpu")
    s = rng.normal(size=(3, 5, 64)).astype(np.float32)
    out["softmax_x"] = s
    out["softmax_out"] = Tensor(s).softmax(axis=-1).numpy(compiler="cpu")
    out["softmax1_out"] = Tensor(s).softmax(axis=1).numpy(compiler="cpu")
    import ml_dtypes
    bf = np.dtype(ml_dtypes.bfloat16)
    x = rng.normal(0, 0.02, size=(3, 2048)).astype(np.float32).astype(bf)
    out["bf16_sumsq_x"] = x.view(np.uint16)
    out["bf16_sumsq_out"] = (Tensor(x) * Tensor(x)).sum(axis=-1, keepdims=True).numpy(
        compiler="cpu").view(np.uint16)
    return out


def generation(ref, workload_name: str, steps: int, keep_logits: tuple, sampling=None,
               prompt_tokens=None, kv_bf16: bool = False) -> dict:
    """Prefill + decode with the reference classes and its cpu compiler.

    Greedy, or with ``sampling = (temperature, top_k, seed)`` each token from
    the reference's own ``sample_native_token`` (generate_tinyllama.py:146-157)
    with ``np.random.default_rng(seed)`` (:712).

    ``kv_bf16``: the plugin's bfloat16 KV-cache mode, through the same graphs
    and compiler.  The reference keeps float32 caches; here every cache it
    returns is rounded to bfloat16 (round to nearest even) before it is bound
    again, and each decode step runs twice: once as usual, which writes the
    new K/V row, then -- after rounding -- again with an all-zero write mask,
    so that the step attends the row as stored (the plugin stores the row it
    writes rounded and attends the stored value).  The second run's logits
    and caches are kept.
    """
    Tensor, compile_graph, get_compiler, no_grad, L = ref
    if sampling is not None:
        from generate_tinyllama import sample_native_token

        temperature, top_k, seed = sampling
        rng = np.random.default_rng(seed)

        def pick(native):
            return sample_native_token(native, temperature=temperature, top_k=top_k, rng=rng, device=device)
    else:
        def pick(native):
            return device.argmax(native)
    from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights
    from cuda_b200.graphs import decode_masks

    wl = WORKLOADS[workload_name]
    cfg = L.LlamaConfig(**{k: getattr(wl.config, k) for k in (
        "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
        "num_attention_heads", "num_key_value_heads", "max_position_embeddings",
        "rms_norm_eps", "rope_theta", "bos_token_id", "eos_token_id")})
    dtype = wl.np_dtype
    device = get_compiler("cpu").device
    weights = {n: Tensor.from_native(v, backend="cpu", shape=v.shape, dtype=v.dtype)
               for n, v in synthetic_weights(wl.config, dtype=dtype).items()}
    prompt = synthetic_prompt(wl.config, prompt_tokens or wl.prompt_tokens)[0]
    context = len(prompt) + steps
    out = {"prompt": prompt, "context": np.int64(context)}
    t0 = time.perf_counter()
    with no_grad():
        model = L.LlamaForCausalLM(cfg, weights, sequence_length=len(prompt), dtype=dtype,
                                   cache_length=context)
        ids = Tensor(prompt.reshape(1, -1).astype(np.int32), copy=False)
        sel = Tensor(L.position_selector(len(prompt) - 1, len(prompt), dtype=dtype), copy=False)
        program = compile_graph(*model.prefill(ids, sel), compiler="cpu", dynamic_inputs=(ids,))
        native = program.run(None, synchronize=False)
        token = pick(native[0])
        out["prefill_logits"] = np.asarray(native[0], dtype=np.float32)
        caches = list(native[1:])
        if kv_bf16:
            caches = [_round_bf16(c) for c in caches]
            out["kv_cache"] = np.array("bfloat16")
        out["prefill_cache_dtype"] = np.array(str(np.asarray(caches[0]).dtype))
        out["prefill_cache_fp"] = np.array([[float(np.sum(np.asarray(c, np.float64))),
                                             float(np.sum(np.abs(np.asarray(c, np.float64))))]
                                            for c in caches])
        print(f"{workload_name}: prefill {time.perf_counter() - t0:.1f}s", flush=True)
        tokens = list(prompt) + [token]
        generated = [token]
        step = L.LlamaDecoderStep(cfg, weights, cache_length=context, dtype=dtype)
        decoder = None
        nodes = None
        top = []
        for i in range(1, steps):
            position = len(tokens) - 1
            host = [np.asarray([[token]], dtype=np.int32),
                    L._rope_rotations(1, cfg.head_size, cfg.rope_theta, dtype, offset=position),
                    *decode_masks(position, context, dtype),
                    np.asarray(position, dtype=np.int32)]
            if decoder is None:
                tensors = [Tensor(v, copy=False) for v in host]
                cts = [Tensor.from_native(v, backend="cpu", shape=tuple(v.shape), dtype=dtype)
                       for v in caches]
                outs = step(tensors[0], tensors[1], tensors[2], tensors[3],
                            list(zip(cts[::2], cts[1::2])), position=tensors[4])
                dyn = [*tensors, *cts]
                decoder = compile_graph(*outs, compiler="cpu", dynamic_inputs=dyn)
                nodes = [t._node for t in dyn]
                bindings = None
            else:
                bindings = dict(zip(nodes, [device.array(v) for v in host] + caches))
            native = decoder.run(bindings, synchronize=False)
            if kv_bf16:  # the written row rounded, then attended as stored (write mask all zero)
                caches = [_round_bf16(c) for c in native[1:]]
                host[3] = np.zeros_like(host[3])
                native = decoder.run(dict(zip(nodes, [device.array(v) for v in host] + caches)),
                                     synchronize=False)
            logits = np.asarray(native[0], dtype=np.float32)
            token = pick(native[0])
            order = np.argsort(-logits[0], kind="stable")[:8]
            top.append(np.stack([order.astype(np.float32), logits[0, order]]))
            if i in keep_logits:
                out[f"step{i}_logits"] = logits
            caches = list(native[1:])
            tokens.append(token)
            generated.append(token)
            if i % 8 == 0:
                print(f"{workload_name}: step {i} {time.perf_counter() - t0:.1f}s", flush=True)
    out["tokens"] = np.asarray(generated, dtype=np.int64)
    out["top8"] = np.asarray(top, dtype=np.float32)
    out["final_cache_fp"] = np.array([[float(np.sum(np.asarray(c, np.float64))),
                                       float(np.sum(np.abs(np.asarray(c, np.float64))))]
                                      for c in caches])
    return out


def _round_bf16(cache):
    """A float32 cache rounded to bfloat16 values (kept as float32, the reference's cache dtype)."""
    import ml_dtypes

    host = np.asarray(cache)
    return host.astype(ml_dtypes.bfloat16).astype(host.dtype)


def sampling_rows(ref) -> dict:
    """The reference's host sampler (generate_tinyllama.py:124-143) on seeded logit rows.

    Rows: N(0, 3) logits, one with a third of its entries -inf (masked), one
    float32 row rounded from bfloat16; per (temperature, top_k) setting the
    token each of a list of seeds gives (a fresh default_rng(seed) per draw).
    """
    from generate_tinyllama import sample_token
    import ml_dtypes

    rng = np.random.default_rng(11)
    width = 2048
    rows = rng.normal(0.0, 3.0, (4, width)).astype(np.float32)
    rows[1, rng.permutation(width)[: width // 3]] = -np.inf
    rows[2] = rows[2].astype(ml_dtypes.bfloat16).astype(np.float32)
    settings = np.array([[0.7, 0], [1.0, 40], [1.5, 1], [0.25, 5], [1.0, width - 1], [2.0, width]], np.float64)
    seeds = np.arange(24, dtype=np.int64) * 7919 + 5
    tokens = np.zeros((rows.shape[0], len(settings), len(seeds)), np.int64)
    for r in range(rows.shape[0]):
        for s, (temperature, top_k) in enumerate(settings):
            for j, seed in enumerate(seeds):
                tokens[r, s, j] = sample_token(rows[r:r + 1], temperature=float(temperature), top_k=int(top_k),
                                               rng=np.random.default_rng(int(seed)))
    return {"rows": rows, "settings": settings, "seeds": seeds, "tokens": tokens}


def block_decode(ref) -> dict:
    """LlamaDecoderBlock vs the same positions, tiny fp32 (pattern of test_llama.py:204-319)."""
    Tensor, compile_graph, get_compiler, no_grad, L = ref
    from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights

    wl = WORKLOADS["tiny-fp32"]
    cfg = L.LlamaConfig(**{k: getattr(wl.config, k) for k in (
        "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
        "num_attention_heads", "num_key_value_heads", "max_position_embeddings")})
    weights = {n: Tensor(v) for n, v in synthetic_weights(wl.config, dtype=np.float32).items()}
    prompt = list(synthetic_prompt(wl.config, 16)[0])
    proposed = [7, 11, 13, 17]
    ctx = len(prompt) + len(proposed)
    pre = L.LlamaForCausalLM(cfg, weights, sequence_length=len(prompt), cache_length=ctx,
                             dtype=np.float32)
    native = compile_graph(*pre.prefill(
        Tensor(np.asarray([prompt], dtype=np.int32), copy=False),
        Tensor(L.position_selector(len(prompt) - 1, len(prompt), dtype=np.float32))),
        compiler="cpu")()
    caches = [(Tensor(native[i]), Tensor(native[i + 1])) for i in range(1, len(native), 2)]
    t = len(proposed)
    start = len(prompt)
    placement = np.zeros((t, ctx), dtype=np.float32)
    placement[np.arange(t), start + np.arange(t)] = 1
    write = placement.sum(axis=0).reshape(1, 1, ctx, 1)
    mask = np.full((1, 1, t, ctx), -1e4, dtype=np.float32)
    for i in range(t):
        mask[0, 0, i, : start + i + 1] = 0
    block = L.LlamaDecoderBlock(cfg, weights, block_length=t, cache_length=ctx, dtype=np.float32)
    got = compile_graph(*block(
        Tensor(np.asarray([proposed], dtype=np.int32), copy=False),
        Tensor(L._rope_rotations(t, cfg.head_size, cfg.rope_theta, np.dtype(np.float32),
                                 offset=start)),
        Tensor(mask), Tensor(placement), Tensor(write), caches), compiler="cpu")()
    return {"prompt": np.asarray(prompt), "proposed": np.asarray(proposed),
            "logits": got[0], "cache0": got[1], "cache_last": got[-1]}


CASES = {
    "six_ops": lambda ref: six_ops(ref),
    "tiny_fp32": lambda ref: generation(ref, "tiny-fp32", 32, (1, 31)),
    "tiny_bf16": lambda ref: generation(ref, "tiny-bf16", 32, (1, 31)),
    "tiny_block": lambda ref: block_decode(ref),
    "tinyllama_bf16": lambda ref: generation(ref, "tinyllama-bf16-bs1", 128, (1, 2, 64, 127)),
    # the Llama-3-8B shape (head size 128, theta 5e5, vocabulary 128256) on two layers
    "llama3_2layer_bf16": lambda ref: generation(ref, "llama3-8b-2layer-bf16", 8, (1, 7)),
    # the bfloat16 KV-cache mode (see generation): TinyLlama shape, 128 steps; Llama-3 shape, 8 steps
    "tinyllama_bf16_kvbf16": lambda ref: generation(ref, "tinyllama-bf16-bs1", 128, (1, 2, 64, 127), kv_bf16=True),
    "llama3_2layer_bf16_kvbf16": lambda ref: generation(ref, "llama3-8b-2layer-bf16", 8, (1, 7), kv_bf16=True),
    # one 2048-token prompt of the prefill workload's length, TinyLlama per-layer shapes on four
    # layers (all 22 would need ~55 GB: the cpu compiler keeps every intermediate): logits, first token
    "tinyllama_prefill2048": lambda ref: generation(ref, "tinyllama-4layer-prefill2048-bf16", 1, ()),
    "sampling": lambda ref: sampling_rows(ref),
    "tiny_fp32_sampled": lambda ref: generation(ref, "tiny-fp32", 32, (), sampling=(0.8, 40, 3)),
}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    parser.add_argument("cases", nargs="*", default=["six_ops", "tiny_fp32", "tiny_bf16", "tiny_block"])
    args = parser.parse_args()
    ref = _reference(args.reference)
    for name in args.cases:
        started = time.perf_counter()
        data = CASES[name](ref)
        np.savez_compressed(HERE / f"{name}.npz", **data)
        print(f"wrote {name}.npz in {time.perf_counter() - started:.1f}s", flush=True)


if __name__ == "__main__":
    main()
