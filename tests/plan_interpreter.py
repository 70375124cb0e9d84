"""NumPy interpreter of ``cuda-b200`` plans -- test infrastructure, not product code.

Executes a :class:`cuda_b200.planner.Plan` on the host: every buffer of the
plan is a flat NumPy array, every step reads and writes the plan's own views
(offsets and strides included), and each step kind computes what the kernel
it launches documents in ``include/chomik_b200.h``:

* ``elementwise`` runs the instruction list with the per-instruction
  rounding; ``reduce`` sums bf16/f16 sequentially with a rounding after
  every add (NumPy's behaviour the kernel repeats);
* ``rms_norm`` and the RMSNorm prologues repeat the staged roundings of
  ``csrc/norm.cuh``; the layer-0 decode norm reads the per-row table of the
  program's ``rms_table`` init step;
* ``gemv`` / ``matmul_multi`` / ``matmul_rows`` apply their x prologue
  (RMSNorm, SwiGLU, table gather) and their epilogue (store, residual,
  SiLU-mul, argmax) around float32 products;
* ``decode_attention`` and ``decode_attention_batched`` rope q and k at the
  bound position from the plan's cos/sin tables, blend k and v into the
  caches where the write mask is non-zero, then attend over the context;
* ``all_reduce`` and ``all_gather`` hand their operand to the caller
  (:func:`run_ranks` sums the ranks' operands, or stacks them, in rank
  order).

The CPU suite runs planned programs through this and compares them with the
parity oracle, so the planner's rewrites (decode fusion, GEMM prologues and
epilogues, the batched attention fusion, tensor-parallel all-reduce steps)
are checked without a GPU.  It fixes the *dataflow*; the kernels' summation
order is not modelled, so comparisons use float tolerances.  Temporary
buffers start as NaN, so a step that reads a value no earlier step wrote
poisons the result, and every view is bounds-checked against its buffer.
"""

from __future__ import annotations

from typing import Dict, Iterator, List, Mapping, Optional, Sequence

import ml_dtypes
import numpy as np

from cuda_b200 import _lib
from cuda_b200.planner import Buffer, Plan, Step, View

BF16 = np.dtype(ml_dtypes.bfloat16)
F32 = np.dtype(np.float32)


def _round(x: np.ndarray, dtype) -> np.ndarray:
    """float32 values rounded to ``dtype`` (a float dtype) and widened back."""
    dtype = np.dtype(dtype)
    if dtype == F32 or dtype.kind not in "fV":
        return np.asarray(x, F32)
    return np.asarray(x, F32).astype(dtype).astype(F32)


def _silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """g / (1 + exp(-g)) * u in float32 steps (llama.py:289-291, :371-380)."""
    with np.errstate(over="ignore"):
        e = np.exp(-g, dtype=F32)
    return ((g / (np.float32(1) + e)) * u).astype(F32)


def _rms(x: np.ndarray, w: np.ndarray, spec, d: Optional[np.ndarray] = None) -> np.ndarray:
    """RMSNorm over the last axis with the reference's staged roundings (csrc/norm.cuh)."""
    sq_dt, sum_dt, mean_dt, t_dt, d_dt, y_dt = spec.dts
    x = np.asarray(x, F32)
    if d is None:
        d = _norm_d(x, spec)
    y = _round(x / d, y_dt)
    return _round(y * np.asarray(w, F32), spec.out_dtype)


def _norm_d(x: np.ndarray, spec) -> np.ndarray:
    """sqrt(mean(x*x) + eps) per row, keepdims (the denominator of the norm)."""
    sq_dt, sum_dt, mean_dt, t_dt, d_dt, _ = spec.dts
    sq = _round(x * x, sq_dt)
    if np.dtype(sum_dt) != F32:  # NumPy's bf16/f16 sum: in order, rounded after each add
        acc = sq[..., 0]
        for i in range(1, sq.shape[-1]):
            acc = _round(acc + sq[..., i], sum_dt)
        s = acc[..., None]
    else:
        s = sq.sum(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    mean = _round(s / np.float32(spec.divisor), mean_dt)
    t = _round(mean + np.float32(spec.eps), t_dt)
    return _round(np.sqrt(t), d_dt)


def _softmax_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray,
                       divisor: float) -> np.ndarray:
    """softmax(q k^T / divisor + mask) v with GQA (q heads grouped over k/v heads)."""
    heads, kvh = q.shape[1], k.shape[1]
    group = heads // kvh
    k = np.repeat(k, group, axis=1)
    v = np.repeat(v, group, axis=1)
    s = np.matmul(q.astype(np.float64), np.swapaxes(k, -1, -2).astype(np.float64)) / divisor + mask
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.matmul(p, v.astype(np.float64)).astype(F32)


class PlanInterpreter:
    """One rank's program state: buffers, and a step-by-step run over them."""

    def __init__(self, plan: Plan, bindings: Optional[Mapping[object, object]] = None) -> None:
        self.plan = plan
        self.bindings = dict(bindings or {})
        self.mem: Dict[int, np.ndarray] = {}
        self.bufs: Dict[int, Buffer] = {}
        for buf in plan.buffers:
            self._flat(buf)

    # ------------------------------------------------------------ memory
    def _flat(self, buf: Buffer) -> np.ndarray:
        flat = self.mem.get(id(buf))
        if flat is not None:
            return flat
        n = max(buf.size, 1)
        if buf.kind == "input":
            value = self.bindings.get(buf.node)
            if value is None:
                value = buf.node.numpy_value()
            value = np.asarray(value)
            if value.shape != tuple(buf.shape):
                raise ValueError(f"{buf.name}: bound shape {value.shape}, plan expects {buf.shape}")
            flat = np.array(value, dtype=buf.dtype).reshape(-1)
            if flat.size == 0:
                flat = np.zeros(1, buf.dtype)
        elif buf.kind == "aux" and buf.host is not None:
            flat = np.array(buf.host, dtype=buf.dtype).reshape(-1)
        elif buf.dtype.kind in "iu" or buf.zero:
            flat = np.zeros(n, buf.dtype)
        else:
            flat = np.full(n, np.nan, dtype=buf.dtype)  # unwritten temporaries poison their readers
        self.mem[id(buf)] = flat
        self.bufs[id(buf)] = buf
        return flat

    def _strided(self, view: View) -> np.ndarray:
        flat = self._flat(view.buf)
        if view.size:
            last = view.offset + sum((n - 1) * s for n, s in zip(view.shape, view.strides) if s > 0)
            first = view.offset + sum((n - 1) * s for n, s in zip(view.shape, view.strides) if s < 0)
            if first < 0 or last >= flat.size:
                raise IndexError(f"view of {view.buf.name} reaches [{first}, {last}] outside {flat.size} elements")
        item = flat.dtype.itemsize
        return np.lib.stride_tricks.as_strided(flat[view.offset:], shape=tuple(view.shape),
                                               strides=tuple(s * item for s in view.strides), writeable=True)

    def read(self, view: View) -> np.ndarray:
        """The view's values as a new array (its dtype)."""
        return np.array(self._strided(view))

    def read_f32(self, view: View) -> np.ndarray:
        return self.read(view).astype(F32)

    def write(self, view: View, value: np.ndarray) -> None:
        target = self._strided(view)
        value = np.asarray(value)
        target[...] = value.reshape(target.shape).astype(view.dtype)

    def buffer_f32(self, buf: Buffer) -> np.ndarray:
        return self._flat(buf).astype(F32)

    # ------------------------------------------------------------ run
    def init(self) -> None:
        for init in self.plan.init_steps:
            if init["name"] != "rms_table":
                raise NotImplementedError(init["name"])
            table = self.read_f32(init["table"])
            d = _norm_d(table, init["spec"])[..., 0]
            self._flat(init["out"])[: d.size] = d

    def steps(self) -> Iterator[Step]:
        """Run the plan; yields each collective step (all_reduce, all_gather) for the caller to complete."""
        self.init()
        for step in self.plan.steps:
            if step.name in COLLECTIVES:
                yield step
                continue
            getattr(self, f"_step_{step.name}")(step)

    def run(self) -> None:
        """Run a plan whose collectives span one rank (the sum or the stack of one operand)."""
        for step in self.steps():
            self.write(step.out, self.read(step.args["src"]))

    def outputs(self) -> List[np.ndarray]:
        outs = []
        for node, view in self.plan.outputs:
            outs.append(self.read(view).reshape(node.shape))
        return outs

    def argmax(self, index: int = 0) -> int:
        return int(self._flat(self.plan.argmax_of[index])[0])

    # ------------------------------------------------------------ generic steps
    def _step_copy(self, step: Step) -> None:
        self.write(step.out, self.read(step.args["src"]))

    def _step_elementwise(self, step: Step) -> None:
        shape = tuple(step.args["shape"])
        regs = [np.broadcast_to(self.read_f32(v), shape) for v in step.args["inputs"]]
        result = None
        with np.errstate(all="ignore"):
            for name, lhs, rhs, dt in step.args["instrs"]:
                a = regs[lhs]
                b = regs[rhs] if rhs >= 0 else None
                if name == "add":
                    r = a + b
                elif name == "sub":
                    r = a - b
                elif name == "mul":
                    r = a * b
                elif name == "div":
                    r = a / b
                elif name == "equal":
                    r = (a == b).astype(F32)
                elif name == "neg":
                    r = -a
                elif name == "exp":
                    r = np.exp(a)
                elif name == "log":
                    r = np.log(a)
                elif name == "sqrt":
                    r = np.sqrt(a)
                elif name == "relu":
                    r = np.maximum(a, np.float32(0))
                elif name == "step":
                    r = (a > 0).astype(F32)
                else:
                    raise NotImplementedError(name)
                result = _round(r, dt)
                regs.append(result)
        self.write(step.out, result)

    def _step_reduce(self, step: Step) -> None:
        src = self.read_f32(step.args["src"])
        keep, red = list(step.args["keep"]), list(step.args["red"])
        moved = np.transpose(src, keep + red)
        kept_shape = moved.shape[:len(keep)]
        flat = moved.reshape(kept_shape + (-1,))
        if step.args["how"] == "max":
            out = flat.max(axis=-1)
        elif step.args["sequential"]:
            acc = flat[..., 0]
            for i in range(1, flat.shape[-1]):
                acc = _round(acc + flat[..., i], step.out.dtype)
            out = acc
        else:
            out = flat.sum(axis=-1, dtype=np.float64)
        self.write(step.out, np.asarray(out).astype(F32))

    def _step_matmul(self, step: Step) -> None:
        a = self.read_f32(step.args["a"])
        b = self.read_f32(step.args["b"])
        self.write(step.out, np.matmul(a.astype(np.float64), b.astype(np.float64)).astype(F32))

    def _step_place(self, step: Step) -> None:
        src = self.read_f32(step.args["src"])
        cols = self._flat(step.args["cols"]).astype(np.int64)
        out = np.zeros(src.shape[:-1] + (cols.size,), F32)
        hit = cols >= 0
        out[..., hit] = src[..., cols[hit]]
        self.write(step.out, out)

    def _step_gather(self, step: Step) -> None:
        table = self.read(step.args["table"])
        idx = self.read(step.args["idx"]).astype(np.int64)
        rows = table.shape[0]
        idx = np.where(idx < 0, idx + rows, idx)
        if np.any((idx < 0) | (idx >= rows)):
            raise IndexError("gather: index outside the table")
        self.write(step.out, table[idx.reshape(-1)])

    def _step_kv_write(self, step: Step) -> None:
        cache_v: View = step.args["cache"]
        cache = self.read_f32(cache_v)
        row = self.read_f32(step.args["row"])
        wm = self.read_f32(step.args["write_mask"]).reshape(-1)
        self.write(cache_v, _blend(cache, row, wm, step.args["one_minus"]))

    # ------------------------------------------------------------ training lowerings
    # what cb_softmax_rows / cb_softmax_backward_rows / cb_layer_norm_rows /
    # cb_layer_norm_backward_rows document, in float32 over rows of `width`
    def _rows(self, view: View, width: int) -> np.ndarray:
        return self.read_f32(view).reshape(-1, width)

    def _step_softmax(self, step: Step) -> None:
        a = step.args
        x = self._rows(a["x"], a["width"])
        shifted = x - x.max(axis=-1, keepdims=True)
        e = np.exp(shifted)
        total = e.sum(axis=-1, keepdims=True)
        self.write(step.out, shifted - np.log(total) if a["log"] else e / total)

    def _step_softmax_backward(self, step: Step) -> None:
        a = step.args
        g, y = self._rows(a["grad"], a["width"]), self._rows(a["y"], a["width"])
        if a["log"]:
            out = g - np.exp(y) * g.sum(axis=-1, keepdims=True)
        else:
            out = y * (g - (g * y).sum(axis=-1, keepdims=True))
        self.write(step.out, out)

    @staticmethod
    def _moments(x: np.ndarray, eps: float):
        mean = x.sum(axis=-1, keepdims=True) / np.float32(x.shape[-1])
        c = x - mean
        return c, np.sqrt((c * c).sum(axis=-1, keepdims=True) / np.float32(x.shape[-1]) + np.float32(eps))

    def _step_layer_norm(self, step: Step) -> None:
        a = step.args
        x = self._rows(a["x"], a["width"])
        c, sd = self._moments(x, a["eps"])
        self.write(step.out, c / sd * self.read_f32(a["w"]) + self.read_f32(a["b"]))

    def _step_layer_norm_backward(self, step: Step) -> None:
        a = step.args
        width = a["width"]
        g, x, w = self._rows(a["grad"], width), self._rows(a["x"], width), self.read_f32(a["w"])
        c, sd = self._moments(x, a["eps"])
        n = c / sd
        if a["dx"] is not None:
            gw = g * w
            self.write(a["dx"], (gw - gw.mean(axis=-1, keepdims=True) - n * (gw * n).mean(axis=-1, keepdims=True))
                       / sd)
        if a["dw"] is not None:
            self.write(a["dw"], (g * n).sum(axis=0))
        if a["db"] is not None:
            self.write(a["db"], g.sum(axis=0))

    def _step_rms_norm(self, step: Step) -> None:
        x = self.read_f32(step.args["x"])
        w = self.read_f32(step.args["w"])
        self.write(step.out, _rms(x, w, step.args["spec"]))

    def _step_rope(self, step: Step) -> None:
        x = self.read_f32(step.args["x"])
        _, _, tokens, hd = x.shape
        offset = 0
        if step.args["offset"] is not None:
            offset = int(self.read(step.args["offset"]).reshape(-1)[0])
        if not 0 <= offset < step.args["n_offsets"]:
            raise IndexError("rope: position outside the table")
        half = hd // 2
        cos = self._flat(step.args["cos"]).reshape(-1, tokens, half)[offset]
        sin = self._flat(step.args["sin"]).reshape(-1, tokens, half)[offset]
        self.write(step.out, _rotate(x, cos, sin))

    def _step_sdpa(self, step: Step) -> None:
        q, k, v, mask = (self.read_f32(step.args[n]) for n in ("q", "k", "v", "mask"))
        out = _softmax_attention(q, k, v, mask.astype(np.float64), step.args["divisor"])
        self.write(step.out, out)

    # ------------------------------------------------------------ GEMMs
    def _prologue(self, args, x: np.ndarray) -> np.ndarray:
        """x (rows, k) after a matmul_multi / matmul_rows x prologue."""
        mode = args["x_mode"]
        if mode == _lib.ROWS_X_RMS:
            return _rms(x, self.read_f32(args["norm_w"]), args["spec"])
        if mode == _lib.ROWS_X_SWIGLU:
            u = self.read_f32(args["x2"]).reshape(x.shape)
            return _silu_mul(x, u)
        return x

    def _products(self, x: np.ndarray, weights: Sequence[View], shapes) -> List[np.ndarray]:
        out = []
        for w, sh in zip(weights, shapes):
            b = self.read_f32(w)
            k, n = b.shape[-2], b.shape[-1]
            out.append(np.matmul(x.astype(np.float64), b.reshape(k, n).astype(np.float64)).astype(F32))
        return out

    def _epilogue(self, step: Step, prods: List[np.ndarray], swiglu: bool) -> None:
        outs: Sequence[View] = step.args["outs"]
        if swiglu:
            self.write(outs[0], _silu_mul(prods[0], prods[1]))
            return
        residual = step.args.get("residual")
        if residual is not None:
            prods = [prods[0] + self.read_f32(residual).reshape(prods[0].shape)]
        for view, value in zip(outs, prods):
            self.write(view, value)

    def _step_matmul_multi(self, step: Step) -> None:
        g = step.args
        x = self.read_f32(g["a"]).reshape(g["m"], g["k"])
        x = self._prologue(g, x)
        prods = self._products(x, g["weights"], g["shapes"])
        self._epilogue(step, prods, g["epilogue"] == _lib.GEMM_SWIGLU)

    def _step_matmul_rows(self, step: Step) -> None:
        g = step.args
        x = self.read_f32(g["x"]).reshape(g["m"], g["k"])
        x = self._prologue(g, x)
        self._epilogue(step, self._products(x, g["weights"], g["shapes"]), False)

    def _step_gemv(self, step: Step) -> None:
        g = step.args
        k = g["k"]
        x_view: View = g["x"]
        if g.get("x_index") is not None:
            table = self.read_f32(x_view)
            row = int(self.read(g["x_index"]).reshape(-1)[0])
            x = table[row % table.shape[0]].reshape(1, k)
        else:
            row = None
            x = self.read_f32(x_view).reshape(1, k)
        spec = g.get("norm")
        if spec is not None:
            d = None
            if g.get("norm_table") is not None:
                d = self._flat(g["norm_table"])[row % self._flat(g["norm_table"]).size].reshape(1, 1)
            x = _rms(x, self.read_f32(g["norm_w"]), spec, d)
        prods = [np.matmul(self.read_f32(w).astype(np.float64), x[0].astype(np.float64)).astype(F32)
                 for w in g["weights"]]
        epi = g["epilogue"]
        if epi == _lib.EPI_SILU_MUL:
            out = _silu_mul(prods[0], prods[1])
        elif epi == _lib.EPI_RESIDUAL:
            res = self.read_f32(g["residual"])
            if g.get("residual_index") is not None:
                rid = int(self.read(g["residual_index"]).reshape(-1)[0])
                res = res[rid % res.shape[0]]
            out = prods[0] + res.reshape(-1)
        else:
            out = np.concatenate(prods)
        self.write(step.out, out)
        if epi == _lib.EPI_ARGMAX:
            self._flat(g["argmax"])[0] = int(np.argmax(out))

    # ------------------------------------------------------------ decode attention
    def _attend_one(self, g, qkv: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                    position: int, wm: np.ndarray, mask: np.ndarray):
        heads, kvh, hd = g["heads"], g["kv_heads"], g["head_size"]
        half = hd // 2
        cos = self._flat(g["cos"]).reshape(g["n_positions"], -1, half)[position, 0]
        sin = self._flat(g["sin"]).reshape(g["n_positions"], -1, half)[position, 0]
        q = qkv[g["q_off"]: g["q_off"] + heads * hd].reshape(1, heads, 1, hd)
        k = qkv[g["k_off"]: g["k_off"] + kvh * hd].reshape(1, kvh, 1, hd)
        v = qkv[g["v_off"]: g["v_off"] + kvh * hd].reshape(1, kvh, 1, hd)
        q, k = _rotate(q, cos[None], sin[None]), _rotate(k, cos[None], sin[None])
        k_cache = _blend(k_cache, k, wm, g["one_minus"])
        v_cache = _blend(v_cache, v, wm, g["one_minus"])
        if g["k_cache"].dtype != F32:  # a bfloat16 cache: the written rows are stored, and attended, rounded
            k_cache = k_cache.astype(g["k_cache"].dtype).astype(F32)
            v_cache = v_cache.astype(g["v_cache"].dtype).astype(F32)
        out = _softmax_attention(q, k_cache, v_cache, mask.reshape(1, 1, 1, -1).astype(np.float64), g["divisor"])
        return out, k_cache, v_cache

    def _position(self, g) -> int:
        position = int(self.read(g["position"]).reshape(-1)[0])
        if not 0 <= position < g["n_positions"]:
            raise IndexError("decode attention: position outside the table")
        return position

    def _step_decode_attention(self, step: Step) -> None:
        g = step.args
        qkv = self.buffer_f32(g["qkv"].buf)
        out, kc, vc = self._attend_one(g, qkv, self.read_f32(g["k_cache"]), self.read_f32(g["v_cache"]),
                                       self._position(g), self.read_f32(g["write_mask"]).reshape(-1),
                                       self.read_f32(g["mask"]))
        self.write(g["k_cache"], kc)
        self.write(g["v_cache"], vc)
        self.write(step.out, out)

    def _step_decode_attention_batched(self, step: Step) -> None:
        g = step.args
        b, row = g["batch"], g["qkv_stride"]
        qkv = self.buffer_f32(g["qkv"].buf)[: b * row].reshape(b, row)
        kc, vc = self.read_f32(g["k_cache"]), self.read_f32(g["v_cache"])
        wm = self.read_f32(g["write_mask"]).reshape(-1)
        mask = self.read_f32(g["mask"])
        position = self._position(g)
        outs = []
        for i in range(b):
            out, kc[i:i + 1], vc[i:i + 1] = self._attend_one(g, qkv[i], kc[i:i + 1], vc[i:i + 1], position, wm, mask)
            outs.append(out)
        self.write(g["k_cache"], kc)
        self.write(g["v_cache"], vc)
        self.write(step.out, np.concatenate(outs, axis=0))


def _rotate(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE over the last axis; cos/sin are (tokens, half) (llama.py:306-323)."""
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    return np.concatenate([lo * cos - hi * sin, lo * sin + hi * cos], axis=-1).astype(F32)


def _blend(cache: np.ndarray, row: np.ndarray, wm: np.ndarray, one_minus) -> np.ndarray:
    """cache*(1-wm) + row*wm at the context rows where wm is non-zero (llama.py:511-512)."""
    cache = cache.copy()
    for r in np.nonzero(wm)[0]:
        w = np.float32(wm[r])
        keep = _round(np.asarray(np.float32(1) - w), one_minus)
        cache[:, :, r, :] = cache[:, :, r, :] * keep + row[:, :, 0, :] * w
    return cache


COLLECTIVES = ("all_reduce", "all_gather")


def run_ranks(interpreters: Sequence[PlanInterpreter]) -> None:
    """Run one plan per rank in lock step: each all_reduce sums the ranks' operands in rank order
    (then adds the step's residual, if it carries one), each all_gather stacks them in rank order."""
    runs = [it.steps() for it in interpreters]
    while True:
        pending = [next(r, None) for r in runs]
        if all(p is None for p in pending):
            return
        if any(p is None for p in pending) or len({p.name for p in pending}) != 1:
            raise RuntimeError("ranks disagree on their collective steps")
        parts = [it.read_f32(p.args["src"]) for it, p in zip(interpreters, pending)]
        if pending[0].name == "all_gather":
            result = np.stack(parts)
        else:
            result = parts[0]
            for part in parts[1:]:
                result = result + part
        for it, p in zip(interpreters, pending):
            residual = p.args.get("residual")
            # an all_reduce carrying the residual add that follows it: hidden + sum
            it.write(p.out, result if residual is None else it.read_f32(residual) + result)
