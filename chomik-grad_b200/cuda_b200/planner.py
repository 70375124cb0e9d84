"""Graph -> kernel plan for the ``cuda-b200`` compiler (host-only, no GPU).

The planner turns a chomik-grad output list into a straight-line list of
kernel launches over a static set of device buffers:

1. **Lowerings.**  Nodes whose intrinsic ``lowering`` the plugin supports
   (``rms_norm``, ``rope``, ``sdpa``; hints attached by chomikgrad/llama.py
   :13-25) are replaced by one kernel, *after* checking that the portable
   sub-graph under the node has the exact shape the reference builds
   (llama.py:279-287, :293-323, :355-364).  The scalar constants of that
   sub-graph (mean divisor, epsilon, attention divisor) and the dtype of
   every intermediate are read from it, so the kernel repeats the arithmetic
   the reference's ``cpu`` compiler performs -- including bfloat16
   intermediates and NumPy's sequential bfloat16 sums.  A lowering whose
   sub-graph does not match is simply not used.
2. **Runtime dtypes.**  Each value gets the dtype NumPy/ml_dtypes would give
   it at run time (bf16 @ bf16 -> float32, bf16 + f32 -> f32, ...), which can
   differ from the node's metadata dtype.
3. **Decode fusion.**  Single-token Llama structures become fused kernels:
   rms_norm -> q/k/v GEMV, RoPE + write-mask cache update + attention,
   O-proj + residual, rms_norm -> gate/up GEMV + SwiGLU, down + residual,
   final norm -> lm_head + argmax.  KV caches bound as dynamic inputs are
   updated in place (the caller rebinds the returned cache,
   generate_tinyllama.py:857).
4. **Generic lowering** of everything else: fused elementwise trees, views
   for RESHAPE/PERMUTE, reductions, batched matmul, gather.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np

from . import _lib

# --------------------------------------------------------------------------
# node helpers (duck-typed: work for the mirror and the real chomikgrad)


def kind(node) -> Optional[str]:
    return None if node.op is None else node.op.value


def is_ew(node, name: Optional[str] = None) -> bool:
    return kind(node) == "elementwise" and (name is None or str(node.arg) == name)


def bf16() -> np.dtype:
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


F32 = np.dtype(np.float32)
FLOATS = ("float32", "bfloat16", "float16")


def dt_code(dtype: np.dtype) -> int:
    return _lib.dtype_code(dtype)


def gemm_shape(step, min_rows: int) -> Optional[Tuple[int, int, int, int, int]]:
    """(m, n, k, lda, ldb) when a MATMUL step is ``x @ W.T`` the tensor-core GEMM takes.

    That is llama.py:275-277 (``inputs @ weight.T``): a bf16 weight seen
    through its transpose (K contiguous), activations whose leading
    dimensions fold into rows, a fresh float32 output, and at least
    ``min_rows`` rows (128-row tiles waste the tensor cores on fewer).
    """
    av = step.args["a"]
    bv = step.args["b"]
    out = step.out
    b16 = bf16()
    if len(av.shape) < 2 or len(bv.shape) < 2 or bv.dtype != b16 or out.dtype != np.float32:
        return None
    if av.dtype not in (np.float32, b16) or not out.is_contiguous():
        return None
    if any(n != 1 for n in bv.shape[:-2]):
        return None
    k, n = bv.shape[-2], bv.shape[-1]
    ldb = bv.strides[-1]
    if bv.strides[-2] != 1 and k > 1:
        return None
    if av.strides[-1] != 1 and k > 1:
        return None
    # every dimension before K folds into rows: the non-unit ones must step by
    # whole rows (a size-1 dimension's stride is meaningless, e.g. the token
    # axis of a permuted single-token attention output)
    dims = [(s, st) for s, st in zip(av.shape[:-1], av.strides[:-1]) if s != 1]
    lda = dims[-1][1] if dims else k
    rows = 1
    for size, stride in reversed(dims):
        if stride != rows * lda:
            return None
        rows *= size
    if rows > 1 and lda < k:  # overlapping or broadcast rows
        return None
    if (rows < min_rows or k % 8 or n % 4 or ldb % 8
            or tuple(out.shape[-2:]) != (av.shape[-2], n)):
        return None
    return rows, n, k, lda, ldb


def contiguous_strides(shape: Sequence[int]) -> Tuple[int, ...]:
    strides, step = [], 1
    for n in reversed(shape):
        strides.append(step)
        step *= max(int(n), 1)
    return tuple(reversed(strides))


class PlanError(TypeError):
    """The graph uses a dtype or construct the plugin cannot run."""


# --------------------------------------------------------------------------
# buffers and views


@dataclass(eq=False)
class Buffer:
    """One device allocation of the program."""

    kind: str                 # input | tmp | aux
    shape: Tuple[int, ...]
    dtype: np.dtype
    node: object = None       # the leaf, for inputs
    name: str = ""
    host: Optional[np.ndarray] = None   # aux: initial contents
    zero: bool = False        # aux: zero-initialised
    bind: str = "copy"        # inputs: copy | pointer (dynamic caches, constants)

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1


@dataclass(eq=False)
class View:
    buf: Buffer
    shape: Tuple[int, ...]
    strides: Tuple[int, ...]
    offset: int = 0

    @property
    def dtype(self) -> np.dtype:
        return self.buf.dtype

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def is_contiguous(self) -> bool:
        expected = contiguous_strides(self.shape)
        return all(n == 1 or s == e for n, s, e in zip(self.shape, self.strides, expected))

    @staticmethod
    def whole(buf: Buffer) -> "View":
        return View(buf, tuple(buf.shape), contiguous_strides(buf.shape), 0)


def reshape_strides(shape: Sequence[int], strides: Sequence[int],
                    new_shape: Sequence[int]) -> Optional[Tuple[int, ...]]:
    """Strides viewing ``shape/strides`` as ``new_shape`` without a copy, or None.

    Same contract as NumPy's no-copy reshape: groups of old axes that are
    contiguous among themselves can be split/merged freely.
    """
    old = [(int(n), int(s)) for n, s in zip(shape, strides) if int(n) != 1]
    new = [int(n) for n in new_shape]
    if int(np.prod([n for n, _ in old], dtype=np.int64)) != int(np.prod(new, dtype=np.int64)):
        return None
    if any(n == 0 for n in new):
        return contiguous_strides(new)
    result = [0] * len(new)
    oi, ni = 0, 0
    # indices of new dims that are not 1
    while ni < len(new) and oi < len(old):
        if new[ni] == 1:
            result[ni] = 0
            ni += 1
            continue
        op, np_ = old[oi][0], new[ni]
        oj, nj = oi + 1, ni + 1
        while op != np_:
            if np_ < op:
                while nj < len(new) and new[nj] == 1:
                    nj += 1
                if nj >= len(new):
                    return None
                np_ *= new[nj]
                nj += 1
            else:
                if oj >= len(old):
                    return None
                op *= old[oj][0]
                oj += 1
        for k in range(oi, oj - 1):
            if old[k][1] != old[k + 1][0] * old[k + 1][1]:
                return None
        stride = old[oj - 1][1]
        for k in range(nj - 1, ni - 1, -1):
            if new[k] == 1:
                result[k] = 0
                continue
            result[k] = stride
            stride *= new[k]
        oi, ni = oj, nj
    while ni < len(new):
        result[ni] = 0
        ni += 1
    return tuple(result)


# --------------------------------------------------------------------------
# steps (one kernel launch each)


@dataclass(eq=False)
class Step:
    name: str
    out: Optional[View]
    args: Dict[str, object] = field(default_factory=dict)
    text: str = ""


# --------------------------------------------------------------------------
# the plan


@dataclass
class RmsSpec:
    divisor: float
    eps: float
    dts: Tuple[np.dtype, ...]  # sq, sum, mean, t, d, y
    out_dtype: np.dtype


class Plan:
    """Result of planning: buffers, steps, outputs and the program source."""

    def __init__(self) -> None:
        self.buffers: List[Buffer] = []
        self.steps: List[Step] = []
        self.leaves: List[object] = []            # all leaves the plan reads
        self.inputs: Tuple[object, ...] = ()      # CompiledProgram.inputs
        self.input_buffers: Dict[object, Buffer] = {}
        self.outputs: List[Tuple[object, View]] = []
        self.aliases: Dict[int, object] = {}      # output index -> dynamic leaf updated in place
        self.argmax_of: Dict[int, Buffer] = {}    # output index -> int64 argmax buffer
        self.error_flag: Optional[Buffer] = None
        self.init_steps: List[dict] = []          # run once when the program is built
        self.guards: List[Tuple[object, np.ndarray]] = []  # non-cached leaves assumed constant
        self.lowered: Dict[str, int] = {}
        self.source = ""

    def buffer(self, kind_: str, shape, dtype, **kw) -> Buffer:
        buf = Buffer(kind_, tuple(int(n) for n in shape), np.dtype(dtype), **kw)
        buf.name = f"{kind_[0]}{len(self.buffers)}"
        self.buffers.append(buf)
        return buf


def _same_table(a, b) -> bool:
    """Whether two constant table buffers hold the same values."""
    if a is b:
        return True
    ha, hb = getattr(a, "host", None), getattr(b, "host", None)
    return ha is not None and hb is not None and ha.shape == hb.shape and bool(np.array_equal(ha, hb))


def _step_reads(step) -> Set[int]:
    """ids of the buffers a step reads (its arguments without its own output list)."""
    acc: Set[int] = set()
    _collect_buffers({k: v for k, v in step.args.items() if k != "outs"}, acc)
    return acc


def _collect_buffers(value, acc: Set[int]) -> None:
    """ids of every Buffer a step argument refers to (Views, lists, dicts)."""
    if isinstance(value, View):
        acc.add(id(value.buf))
    elif isinstance(value, Buffer):
        acc.add(id(value))
    elif isinstance(value, (list, tuple)):
        for v in value:
            _collect_buffers(v, acc)
    elif isinstance(value, dict):
        for v in value.values():
            _collect_buffers(v, acc)


class Planner:
    """Builds a :class:`Plan` from output nodes (see module docstring)."""

    SUPPORTED_LOWERINGS = frozenset({"rms_norm", "rope", "sdpa", "all_reduce", "all_gather",
                                     "softmax", "log_softmax", "softmax_backward", "log_softmax_backward",
                                     "layer_norm", "layer_norm_backward"})
    # the training lowerings' hinted subgraphs end in these operations (chomikgrad/tensor.py:316-450)
    _TRAIN_TOP = {"softmax": "div", "log_softmax": "sub", "softmax_backward": "mul",
                  "log_softmax_backward": "sub", "layer_norm": "add"}

    def __init__(self, outputs: Sequence[object], dynamic_inputs: Sequence[object], *,
                 backend: str, leaf_dtype, max_positions: int = 8192,
                 fuse_decode: bool = True, alias_caches: bool = True,
                 table_cache: Optional[dict] = None, gemm_min_rows: Optional[int] = None,
                 kv_bf16: bool = False) -> None:
        self.outputs = tuple(outputs)
        self.dynamic = set(dynamic_inputs)
        self.backend = backend
        self.leaf_dtype = leaf_dtype
        self.max_positions = max_positions
        self.fuse_decode = fuse_decode
        self.alias_caches = alias_caches
        self.table_cache = table_cache if table_cache is not None else {}
        self.gemm_min_rows = gemm_min_rows  # None: no tensor-core GEMM epilogue fusion
        # bfloat16 KV caches: the prefill's cache placement stores bfloat16, and the
        # fused decode attentions accept bfloat16 caches (rows they write are rounded)
        self.kv_bf16 = kv_bf16
        self.plan = Plan()
        self._rdt: Dict[object, np.dtype] = {}
        self._val: Dict[object, View] = {}
        self._low: Dict[object, Tuple[str, tuple, object]] = {}
        self._rms: Dict[object, RmsSpec] = {}
        self._sdpa: Dict[object, float] = {}
        self._rope: Dict[object, object] = {}
        self.units: Dict[object, object] = {}

    # ---------------------------------------------------------------- dtypes
    def rdt(self, node) -> np.dtype:
        """Runtime dtype NumPy/ml_dtypes produce for ``node`` (iterative)."""
        if node in self._rdt:
            return self._rdt[node]
        stack = [node]
        while stack:
            top = stack[-1]
            if top in self._rdt:
                stack.pop()
                continue
            pending = [p for p in top.inputs if p not in self._rdt]
            if pending:
                stack.extend(pending)
                continue
            stack.pop()
            self._rdt[top] = self._infer(top)
        return self._rdt[node]

    def _infer(self, node) -> np.dtype:
        k = kind(node)
        if k is None:
            return np.dtype(self.leaf_dtype(node))
        ins = [self._rdt[p] for p in node.inputs]
        if k == "elementwise":
            name = str(node.arg)
            if name == "equal":
                return ins[0]
            if len(ins) == 2:
                return np.result_type(ins[0], ins[1])
            return ins[0]
        if k == "matmul":
            if ins[0].name == "bfloat16" and ins[1].name == "bfloat16":
                return F32
            return np.result_type(ins[0], ins[1])
        if k in ("reshape", "permute", "reduce"):
            return ins[0]
        if k == "gather":
            return ins[0]
        raise PlanError(f"unsupported operation: {node.op}")

    # ------------------------------------------------------- graph analysis
    def _lowering_of(self, node):
        low = node.lowering
        if low is None or low[0] not in self.SUPPORTED_LOWERINGS:
            return None
        kind_ = low[0]
        if kind_ == "rms_norm" and self._match_rms(node, low):
            return low
        if kind_ == "rope" and self._match_rope(node, low):
            return low
        if kind_ == "sdpa" and self._match_sdpa(node, low):
            return low
        if kind_ == "all_reduce" and self._match_all_reduce(node, low):
            return low
        if kind_ == "all_gather" and self._match_all_gather(node, low):
            return low
        if kind_ in self._TRAIN_TOP or kind_ == "layer_norm_backward":
            return low if self._match_train(node, low) else None
        return None

    def _match_train(self, node, low) -> bool:
        """The training lowerings (softmax / log_softmax and their backward, layer_norm and its
        backward), float32 over the last axis.  The reference builds the hinted subgraph and
        the hint together (chomikgrad/tensor.py:316-450); the checks here are the ones the
        kernels rely on: dtypes, shapes, the axis, the subgraph's final operation."""
        name, inputs, arg = low[0], low[1], low[2]
        if any(self.rdt(n) != F32 for n in (node, *inputs)) or not node.shape:
            return False
        width = node.shape[-1] if name != "layer_norm_backward" else inputs[1].shape[-1]
        if name in self._TRAIN_TOP:
            if not is_ew(node, self._TRAIN_TOP[name]):
                return False
            if name in ("softmax", "log_softmax", "softmax_backward", "log_softmax_backward"):
                return (arg == len(node.shape) - 1 and all(tuple(n.shape) == tuple(node.shape) for n in inputs))
            x, w, b = inputs
            return (tuple(x.shape) == tuple(node.shape) and tuple(w.shape) == (width,)
                    and tuple(b.shape) == (width,) and float(arg) > 0)
        grad, x, w = inputs
        if not (isinstance(arg, tuple) and len(arg) == 2 and arg[1] in (0, 1, 2) and float(arg[0]) > 0):
            return False
        if tuple(grad.shape) != tuple(x.shape) or tuple(w.shape) != (width,):
            return False
        return tuple(node.shape) == (tuple(x.shape) if arg[1] == 0 else (width,))

    def _parents(self, node):
        low = self._low.get(node)
        return low[1] if low is not None else node.inputs

    def _order(self) -> List[object]:
        order, seen = [], set()
        for root in self.outputs:
            if root in seen:
                continue
            seen.add(root)
            stack = [(root, None)]
            while stack:
                node, it = stack[-1]
                if it is None:
                    low = self._lowering_of(node) if node.op is not None else None
                    if low is not None:
                        self._low[node] = low
                    it = iter(self._parents(node))
                    stack[-1] = (node, it)
                advanced = False
                for parent in it:
                    if parent not in seen:
                        seen.add(parent)
                        stack.append((parent, None))
                        advanced = True
                        break
                if not advanced:
                    stack.pop()
                    order.append(node)
        return order

    # --- structural matchers of the reference's portable sub-graphs -------
    def _const(self, node) -> Optional[float]:
        """Value of a constant scalar leaf (immutable: cached native)."""
        if node.op is not None or node in self.dynamic or not node.cache_native:
            return None
        if int(np.prod(node.shape)) != 1:
            return None
        try:
            value = np.asarray(node.numpy_value())
        except Exception:
            return None
        return float(value.reshape(-1)[0].astype(np.float32))

    def _match_all_reduce(self, node, low) -> bool:
        """out = x * 1: the portable form of a tensor-parallel sum (cuda_b200.tensor_parallel)."""
        if not is_ew(node, "mul") or len(low[1]) != 1 or not isinstance(low[2], str):
            return False
        x = low[1][0]
        if len(node.inputs) != 2 or node.inputs[0] is not x or self._const(node.inputs[1]) != 1.0:
            return False
        return self.rdt(x).name in ("float32", "bfloat16")

    def _match_all_gather(self, node, low) -> bool:
        """out = x.reshape(1, *x.shape) * ones(G, 1, ..., 1): the portable form of a
        tensor-parallel gather of G shards (cuda_b200.tensor_parallel); exact on one rank."""
        if not is_ew(node, "mul") or len(low[1]) != 1 or not isinstance(low[2], str) or len(node.inputs) != 2:
            return False
        x = low[1][0]
        spread, ones = node.inputs
        if kind(spread) != "reshape" or spread.inputs[0] is not x or tuple(spread.shape) != (1,) + tuple(x.shape):
            return False
        if ones.op is not None or ones in self.dynamic:
            return False
        if tuple(ones.shape) != (node.shape[0],) + (1,) * len(x.shape):
            return False
        try:
            value = np.asarray(ones.numpy_value())
        except Exception:
            return False
        if not np.all(value == 1) or self.rdt(x).name not in ("float32", "bfloat16") or self.rdt(node) != self.rdt(x):
            return False
        if not ones.cache_native:  # specialised on: checked again before every run
            self.plan.guards.append((ones, value.copy()))
        return True

    def _match_rms(self, node, low) -> bool:
        """out = x / sqrt(sum(x*x, -1, keepdims)/c + eps) * w (llama.py:279-287)."""
        x, w = low[1]
        if not is_ew(node, "mul") or node.inputs[1] is not w:
            return False
        a = node.inputs[0]
        if not is_ew(a, "div") or a.inputs[0] is not x:
            return False
        s = a.inputs[1]
        if not is_ew(s, "sqrt"):
            return False
        t = s.inputs[0]
        if not is_ew(t, "add"):
            return False
        m, e = t.inputs
        if not is_ew(m, "div"):
            return False
        total, c = m.inputs
        if kind(total) != "reduce":
            return False
        how, axes, keep = total.arg
        if how != "sum" or tuple(axes) != (len(x.shape) - 1,) or not keep:
            return False
        q = total.inputs[0]
        if not is_ew(q, "mul") or q.inputs[0] is not x or q.inputs[1] is not x:
            return False
        divisor, eps = self._const(c), self._const(e)
        if divisor is None or eps is None or len(w.shape) != 1 or w.shape[0] != x.shape[-1]:
            return False
        # the constants enter the arithmetic in their own runtime dtype
        divisor = float(np.asarray(divisor, dtype=np.float32).astype(self.rdt(c)).astype(np.float32))
        eps = float(np.asarray(eps, dtype=np.float32).astype(self.rdt(e)).astype(np.float32))
        dts = tuple(self.rdt(n) for n in (q, total, m, t, s, a))
        if any(d.name not in FLOATS for d in dts) or self.rdt(node).name not in FLOATS:
            return False
        self._rms[node] = RmsSpec(divisor, eps, dts, self.rdt(node))
        return True

    def _match_rope(self, node, low) -> bool:
        """out = reshape(reshape(x) @ R) with R (1,1,T,hd,hd) (llama.py:293-323)."""
        inputs, (hd, theta, offset) = low[1], low[2]
        x = inputs[0]
        if kind(node) != "reshape" or len(x.shape) != 4:
            return False
        mm = node.inputs[0]
        if kind(mm) != "matmul" or kind(mm.inputs[0]) != "reshape" or mm.inputs[0].inputs[0] is not x:
            return False
        rot = mm.inputs[1]
        b, h, t, d = x.shape
        if d != hd or d % 2 or rot.op is not None or tuple(rot.shape) != (1, 1, t, d, d):
            return False
        if self.rdt(node).name not in FLOATS or int(offset) != 0:
            return False
        position = inputs[1] if len(inputs) == 2 else None
        if position is None:
            # constant rotation table: read cos/sin straight from it
            if rot in self.dynamic or not rot.cache_native:
                return False
            table = np.asarray(rot.numpy_value()).astype(np.float32)[0, 0]
            half = d // 2
            j = np.arange(half)
            cos = table[:, j, j][None]          # [1][T][half]
            sin = table[:, j, j + half][None]
            self._rope[node] = ("table", cos.copy(), sin.copy())
        else:
            if position.shape != () or np.dtype(self.rdt(position)).kind not in "iu":
                return False
            self._rope[node] = ("position", float(theta), self.rdt(rot), t, d)
        return True

    def _repeat_source(self, node, heads: int):
        """k for reshape(reshape(k) * ones(1,1,G,1,1)) (llama.py:325-330), else None."""
        if kind(node) != "reshape":
            return None
        mul = node.inputs[0]
        if not is_ew(mul, "mul"):
            return None
        inner, ones = mul.inputs
        if kind(inner) != "reshape" or ones.op is not None or ones in self.dynamic:
            return None
        src = inner.inputs[0]
        if len(src.shape) != 4:
            return None
        b, kvh, t, d = src.shape
        if tuple(inner.shape) != (b, kvh, 1, t, d) or kvh == 0 or heads % kvh:
            return None
        if tuple(ones.shape) != (1, 1, heads // kvh, 1, 1):
            return None
        try:
            ones_value = np.asarray(ones.numpy_value())
        except Exception:
            return None
        if not np.all(ones_value == 1):
            return None
        if not ones.cache_native:
            self.plan.guards.append((ones, ones_value.copy()))
        return src

    def _match_sdpa(self, node, low) -> bool:
        """out = softmax((q @ rep(k)^T) / c + mask) @ rep(v) (llama.py:355-364)."""
        q, k, v, mask = low[1]
        if kind(node) != "matmul" or len(q.shape) != 4:
            return False
        heads = q.shape[1]
        probs, rep_v = node.inputs
        if self._repeat_source(rep_v, heads) is not v:
            return False
        # softmax portable form: div(exp(sub(x, max)), sum(...)), hint ("softmax", (x,), axis)
        slow = probs.lowering
        if slow is None or slow[0] != "softmax" or int(slow[2]) != 3:
            return False
        scores = slow[1][0]
        if not is_ew(scores, "add") or scores.inputs[1] is not mask:
            return False
        scaled = scores.inputs[0]
        if not is_ew(scaled, "div"):
            return False
        qk, c = scaled.inputs
        if kind(qk) != "matmul" or qk.inputs[0] is not q:
            return False
        kt = qk.inputs[1]
        if kind(kt) != "permute" or tuple(kt.arg) != (0, 1, 3, 2):
            return False
        if self._repeat_source(kt.inputs[0], heads) is not k:
            return False
        divisor = self._const(c)
        if divisor is None or len(mask.shape) != 4:
            return False
        divisor = float(np.asarray(divisor, dtype=np.float32).astype(self.rdt(c)).astype(np.float32))
        if any(self.rdt(n) != F32 for n in (scaled, scores, probs, node)):
            return False
        self._sdpa[node] = divisor
        return True

    # ------------------------------------------------------------ planning
    def build(self) -> Plan:
        plan = self.plan
        order = self._order()
        self.order = order
        for node in order:
            dt = self.rdt(node)
            if node.op is not None and dt.name not in FLOATS + ("int32", "int64"):
                raise PlanError(f"cuda-b200 does not support runtime dtype {dt} "
                                f"(node {kind(node)} {node.arg!r})")
        leaves = [n for n in order if n.op is None]
        if not self.dynamic.issubset(set(leaves) | self._pruned_leaves()):
            raise ValueError("dynamic input is not a leaf of the compiled graph")
        plan.leaves = leaves
        plan.dynamic = set(self.dynamic)
        plan.inputs = tuple(n for n in leaves if n in self.dynamic) if self.dynamic else tuple(leaves)
        self.consumers: Dict[object, List[object]] = {}
        for node in order:
            for parent in self._parents(node):
                self.consumers.setdefault(parent, []).append(node)
        self.output_set = set(self.outputs)
        self.claimed: Set[object] = set()
        for leaf in leaves:
            self._bind_leaf(leaf)
        if self.fuse_decode:
            from .fusion import DecodeFusion

            DecodeFusion(self).apply()
        if self.alias_caches:
            self._match_kv_writes()
        self._match_all_reduce_adds()
        self._fuse_elementwise_groups()
        for node in order:
            if node.op is None or node in self._val:
                continue
            unit = self.units.get(node)
            if unit is not None:
                unit()
            elif node not in self.claimed:
                self._emit_generic(node)
        for index, node in enumerate(self.outputs):
            plan.outputs.append((node, self.value(node)))
        self._drop_dead_steps()  # before the fusion: dead copies must not count as readers
        self._fuse_gemms()
        self._drop_dead_steps()
        from .fusion import assign_prefetch

        assign_prefetch(plan.steps)
        plan.source = self._source()
        return plan

    def _match_kv_writes(self) -> None:
        """``cache*(1-wm) + row*wm`` on a dynamic cache (llama.py:511-512) => in-place cb_kv_write.

        For caches of any batch (the batch-1 decode fusion claims its own
        first): the cache leaf is bound by pointer, updated in place and
        returned as the same object, like the reference runtime rebinding
        the returned caches as the next step's inputs.
        """
        for node in self.order:
            if not is_ew(node, "add") or node not in self.output_set or node in self.claimed or node in self.units:
                continue
            left, right = node.inputs
            if not (is_ew(left, "mul") and is_ew(right, "mul")):
                continue
            cache, keep = left.inputs
            row, wm = right.inputs
            if not is_ew(keep, "sub") or keep.inputs[1] is not wm or self._const(keep.inputs[0]) != 1.0:
                continue
            if (cache.op is not None or cache not in self.dynamic or cache in self.output_set
                    or len(cache.shape) != 4 or self.rdt(cache) not in self.kv_dtypes()):
                continue
            b, h, ctx, hd = cache.shape
            if tuple(row.shape) != (b, h, 1, hd) or tuple(wm.shape) != (1, 1, ctx, 1):
                continue
            if (self.rdt(wm).name not in FLOATS or self.rdt(left) not in self.kv_dtypes()
                    or any(self.rdt(n) != F32 for n in (right, node, row))):
                continue
            uses = self.consumers
            if not (len(uses.get(cache, ())) == 1 and uses.get(left) == [node] and uses.get(right) == [node]
                    and uses.get(keep) == [left]):
                continue
            self.claimed.update((left, right, keep))
            self.units[node] = self._kv_write_unit(node, cache, row, wm, keep)

    def _match_all_reduce_adds(self) -> None:
        """``hidden + all_reduce(partial)`` (the residual add after the row-sharded O and down
        projections, llama.py:526-535 over shards) => one all_reduce step carrying the residual:
        the peer kernel adds it while it sums the ranks' partials (NCCL's path adds it after)."""
        for node in self.order:
            if not is_ew(node, "add") or node in self.claimed or node in self.units or node in self._low:
                continue
            for reduced, other in ((node.inputs[1], node.inputs[0]), (node.inputs[0], node.inputs[1])):
                low = self._low.get(reduced)
                if low is None or low[0] != "all_reduce" or reduced in self.output_set:
                    continue
                if self.consumers.get(reduced) != [node] or tuple(reduced.shape) != tuple(node.shape):
                    continue
                if tuple(other.shape) != tuple(node.shape) or self.rdt(node) != F32 or self.rdt(reduced) != F32:
                    continue
                if self.rdt(other).name not in ("float32", "bfloat16") or self.rdt(low[1][0]) != F32:
                    continue
                self.claimed.add(reduced)
                self.units[node] = self._all_reduce_add_unit(node, reduced, low, other)
                break

    def _all_reduce_add_unit(self, node, reduced, low, other):
        def emit() -> None:
            src = self.contiguous(self.value(low[1][0]))
            res = self.contiguous(self.value(other))
            out = self.tmp(node.shape, F32)
            self.plan.lowered["all_reduce"] = self.plan.lowered.get("all_reduce", 0) + 1
            self.add_step("all_reduce", out, f"{self._name(res)} + all_reduce({self._name(src)}, group={low[2]!r})",
                          src=src, group=low[2], flag=self.error_flag(), residual=res)
            self.set_value(node, out)
        return emit

    def kv_dtypes(self) -> Tuple[np.dtype, ...]:
        """Cache dtypes the decode blends accept: float32, and bfloat16 in bfloat16-KV mode."""
        return (F32, bf16()) if self.kv_bf16 else (F32,)

    def _kv_write_unit(self, node, cache, row, wm, keep):
        def emit() -> None:
            view = self.value(cache)
            view.buf.bind = "pointer"
            rv, wv = self.value(row), self.contiguous(self.value(wm))
            self.add_step("kv_write", view, f"kv_write({self._name(view)}, {self._name(rv)}, "
                          f"write_mask={self._name(wv)}) (in place)",
                          cache=view, row=rv, write_mask=wv, one_minus=self.rdt(keep))
            self.set_value(node, view)
            for i, o in enumerate(self.outputs):
                if o is node:
                    self.plan.aliases[i] = cache
        return emit

    # steps whose only effect is their output buffer
    # ------------------------------------------------ GEMM epilogue fusion
    _SWIGLU = [("neg", 0, -1), ("exp", 3, -1), ("add", 4, 1), ("div", 0, 5), ("mul", 6, 2)]

    def _fuse_gemms(self) -> None:
        """Fold the prefill's tensor-core GEMMs and their elementwise neighbours.

        On steps whose matmuls run on cb_gemm_tc (``gemm_shape`` with the
        compiler's row threshold), three rewrites into ``matmul_multi`` steps
        (cb_gemm_tc_multi):
        * SwiGLU: ``silu(x @ Wg.T) * (x @ Wu.T)`` -- the reference's
          elementwise chain g / (1 + exp(-g)) * u (llama.py:289-291) over two
          matmuls of the same x read by nothing else -- becomes one launch
          whose epilogue computes the chain (same float32 steps);
        * residual: ``r + x @ W.T`` (llama.py:529-535) with a float32 r
          computed before the matmul becomes the GEMM's epilogue add;
        * grouping: up to three remaining matmuls of the same x (q/k/v)
          become one launch.
        Each removed matmul output was read by the fused elementwise step
        only, so no other step sees a difference.
        """
        if self.gemm_min_rows is None:
            return
        plan = self.plan
        steps = plan.steps
        readers: Dict[int, int] = {}
        for st in steps:
            acc: Set[int] = set()
            _collect_buffers(st.args, acc)
            for b in acc:
                readers[b] = readers.get(b, 0) + 1
        external = {id(v.buf) for _, v in plan.outputs} | {id(b) for b in plan.argmax_of.values()}
        producer = {id(st.out.buf): st for st in steps if st.out is not None}
        index = {id(st): i for i, st in enumerate(steps)}
        removed: Set[int] = set()
        replace: Dict[int, Step] = {}

        def gemmable(st) -> Optional[tuple]:
            if st is None or st.name != "matmul" or id(st) in removed or id(st) in replace:
                return None
            return gemm_shape(st, self.gemm_min_rows)

        def only_for(view: View, consumer) -> Optional[Step]:
            """The matmul producing all of ``view``'s buffer, read by ``consumer`` alone."""
            st = producer.get(id(view.buf))
            if st is None or readers.get(id(view.buf), 0) != 1 or id(view.buf) in external:
                return None
            if view.offset != 0 or not view.is_contiguous() or view.size != view.buf.size:
                return None
            return st

        def same_a(x: Step, y: Step) -> bool:
            a, b = x.args["a"], y.args["a"]
            return a.buf is b.buf and a.offset == b.offset and a.shape == b.shape and a.strides == b.strides

        def fused(first: Step, mats: List[Step], epilogue: int, outs: List[View], residual=None) -> Step:
            m, _, k, lda, _ = gemm_shape(first, self.gemm_min_rows)
            args = dict(a=first.args["a"], weights=[st.args["b"] for st in mats],
                        shapes=[gemm_shape(st, self.gemm_min_rows) for st in mats], outs=outs,
                        epilogue=epilogue, residual=residual, m=m, k=k, lda=lda, x_mode=_lib.ROWS_X_PLAIN,
                        norm_w=None, spec=None)
            names = ", ".join(self._name(st.args["b"]) for st in mats)
            kind_ = {_lib.GEMM_STORE: "store", _lib.GEMM_RESIDUAL: "residual", _lib.GEMM_SWIGLU: "swiglu"}[epilogue]
            text = f"matmul_multi({self._name(first.args['a'])}, [{names}], epilogue={kind_})"
            return Step("matmul_multi", outs[0], args, text)

        for st in steps:  # SwiGLU and residual epilogues
            if st.name != "elementwise" or id(st) in removed:
                continue
            ins, ops = st.args["inputs"], st.args["instrs"]
            if any(np.dtype(o[3]) != np.float32 for o in ops) or st.out.dtype != np.float32:
                continue
            shape = tuple(st.out.shape)
            if len(ins) == 3 and [tuple(o[:3]) for o in ops] == self._SWIGLU:
                one = ins[1]
                if one.buf.kind != "input" or one.buf.node is None or self._const(one.buf.node) != 1.0:
                    continue
                g, u = only_for(ins[0], st), only_for(ins[2], st)
                if (g is None or u is None or g is u or tuple(ins[0].shape) != shape or tuple(ins[2].shape) != shape
                        or not same_a(g, u)):
                    continue
                sg, su = gemmable(g), gemmable(u)
                if sg is None or su is None or sg[0] != su[0] or sg[1] != su[1] or sg[2:4] != su[2:4]:
                    continue
                first, second = (g, u) if index[id(g)] < index[id(u)] else (u, g)
                replace[id(first)] = fused(g, [g, u], _lib.GEMM_SWIGLU, [st.out])
                removed.update((id(second), id(st)))
            elif len(ins) == 2 and [tuple(o[:3]) for o in ops] == [("add", 0, 1)]:
                for mi, ri in ((1, 0), (0, 1)):
                    mat = only_for(ins[mi], st)
                    r = ins[ri]
                    if mat is None or gemmable(mat) is None or tuple(ins[mi].shape) != shape:
                        continue
                    if r.dtype != np.float32 or tuple(r.shape) != shape or not r.is_contiguous():
                        continue
                    made = producer.get(id(r.buf))
                    if made is not None and index[id(made)] > index[id(mat)]:
                        continue  # the residual is computed after the matmul
                    replace[id(mat)] = fused(mat, [mat], _lib.GEMM_RESIDUAL, [st.out], residual=r)
                    removed.add(id(st))
                    break
        for i, st in enumerate(steps):  # group plain matmuls that share x
            if gemmable(st) is None:
                continue
            group = [st]
            written = set()
            for later in steps[i + 1:]:
                if len(group) == 3:
                    break
                if later.out is not None:
                    written.add(id(later.out.buf))
                if id(st.args["a"].buf) in written:
                    break
                if (gemmable(later) is not None and same_a(st, later)
                        and gemm_shape(later, self.gemm_min_rows)[2:4] == gemm_shape(st, self.gemm_min_rows)[2:4]):
                    group.append(later)
            if len(group) > 1:
                replace[id(st)] = fused(st, group, _lib.GEMM_STORE, [g.out for g in group])
                removed.update(id(g) for g in group[1:])
        plan.steps = [replace.get(id(st), st) for st in steps if id(st) not in removed]
        self._fuse_norm_into_gemm()
        self._fuse_rows()

    def _fuse_norm_into_gemm(self) -> None:
        """An RMSNorm read by one tensor-core GEMM step only becomes its A prologue.

        cb_gemm_tc_multi computes rms_norm(x) * w (the same rounding stages)
        while it splits A into bf16 planes, so the normalised activations are
        never stored.
        """
        plan = self.plan
        readers: Dict[int, List[Step]] = {}
        for st in plan.steps:
            acc: Set[int] = set()
            _collect_buffers(st.args, acc)
            for b in acc:
                readers.setdefault(b, []).append(st)
        external = {id(v.buf) for _, v in plan.outputs} | {id(b) for b in plan.argmax_of.values()}
        removed: Set[int] = set()
        for st in plan.steps:
            if st.name != "rms_norm" or st.args.get("table") is not None or id(st.out.buf) in external:
                continue
            users = readers.get(id(st.out.buf), [])
            if len(users) != 1 or users[0].name != "matmul_multi" or users[0].args["x_mode"] != _lib.ROWS_X_PLAIN:
                continue
            mm, x = users[0], st.args["x"]
            a = mm.args["a"]
            if (a.buf is not st.out.buf or a.offset != 0 or not a.is_contiguous() or not x.is_contiguous()
                    or x.dtype not in (np.float32, bf16()) or st.out.dtype not in (np.float32, bf16())
                    or tuple(x.shape) != tuple(st.out.shape)):
                continue
            mm.args.update(a=x, lda=x.shape[-1], x_mode=_lib.ROWS_X_RMS, norm_w=st.args["w"], spec=st.args["spec"])
            mm.text = mm.text[:-1] + ", prologue=rms_norm)"
            removed.add(id(st))
        plan.steps = [st for st in plan.steps if id(st) not in removed]

    def _rows_route(self, st) -> Optional[tuple]:
        """gemm_shape of a matmul that runs on cb_gemm_rows (few rows, dense weight rows)."""
        if st.name != "matmul":
            return None
        shape = gemm_shape(st, 1)
        if shape is None or shape[0] >= self.gemm_min_rows or shape[0] > 256 or shape[4] != shape[2]:
            return None
        return shape

    def _fuse_rows(self) -> None:
        """Fold batched decode's elementwise neighbours into cb_gemm_rows (``matmul_rows`` steps).

        * RMSNorm read only by up to three row-GEMM matmuls of its output
          (q/k/v, gate/up) becomes their x prologue (the norm is computed
          while x is split into bf16 planes);
        * SwiGLU read only by one row-GEMM matmul (down) becomes its prologue;
        * ``r + x @ W.T`` with a float32 r computed before becomes the
          residual epilogue of a one-weight row GEMM.
        """
        plan = self.plan
        steps = plan.steps
        readers: Dict[int, List[Step]] = {}
        for st in steps:
            acc: Set[int] = set()
            _collect_buffers(st.args, acc)
            for b in acc:
                readers.setdefault(b, []).append(st)
        external = {id(v.buf) for _, v in plan.outputs} | {id(b) for b in plan.argmax_of.values()}
        producer = {id(st.out.buf): st for st in steps if st.out is not None}
        index = {id(st): i for i, st in enumerate(steps)}
        removed: Set[int] = set()
        replace: Dict[int, Step] = {}

        def sole_readers(st) -> Optional[List[Step]]:
            buf = st.out.buf
            if id(buf) in external or st.out.offset != 0 or not st.out.is_contiguous():
                return None
            return readers.get(id(buf), [])

        def rows_step(x: View, mats: List[Step], shapes, outs, **extra) -> Step:
            m, _, k, ldx, _ = shapes[0]
            args = dict(x=x, weights=[st.args["b"] for st in mats], shapes=shapes, outs=outs, m=m, k=k,
                        ldx=ldx, x_mode=extra.get("x_mode", _lib.ROWS_X_PLAIN), norm_w=extra.get("norm_w"),
                        spec=extra.get("spec"), x2=extra.get("x2"), residual=extra.get("residual"))
            names = ", ".join(self._name(st.args["b"]) for st in mats)
            mode = {_lib.ROWS_X_PLAIN: "", _lib.ROWS_X_RMS: ", prologue=rms_norm",
                    _lib.ROWS_X_SWIGLU: ", prologue=swiglu"}[args["x_mode"]]
            res = ", epilogue=residual" if args["residual"] is not None else ""
            return Step("matmul_rows", outs[0], args, f"matmul_rows({self._name(x)}, [{names}]{mode}{res})")

        for st in steps:  # RMSNorm prologues
            if st.name != "rms_norm" or st.args.get("table") is not None:
                continue
            users = sole_readers(st)
            if not users or len(users) > 3 or any(self._rows_route(u) is None for u in users):
                continue
            shapes = [self._rows_route(u) for u in users]
            if (any(u.args["a"].buf is not st.out.buf or u.args["a"].offset != 0 for u in users)
                    or len({sh[2:4] for sh in shapes}) != 1 or shapes[0][3] != shapes[0][2]):
                continue
            x = st.args["x"]
            if not x.is_contiguous() or x.dtype not in (np.float32, bf16()):
                continue
            first = min(users, key=lambda u: index[id(u)])
            shapes_x = [(sh[0], sh[1], sh[2], x.shape[-1], sh[4]) for sh in shapes]
            replace[id(first)] = rows_step(x, users, shapes_x, [u.out for u in users], x_mode=_lib.ROWS_X_RMS,
                                           norm_w=st.args["w"], spec=st.args["spec"])
            removed.update(id(u) for u in users if u is not first)
            removed.add(id(st))
        for st in steps:  # SwiGLU prologues
            if st.name != "elementwise" or id(st) in removed:
                continue
            ins, ops = st.args["inputs"], st.args["instrs"]
            if ([tuple(o[:3]) for o in ops] != self._SWIGLU or any(np.dtype(o[3]) != np.float32 for o in ops)
                    or ins[1].buf.kind != "input" or ins[1].buf.node is None
                    or self._const(ins[1].buf.node) != 1.0):
                continue
            users = sole_readers(st)
            if not users or len(users) != 1 or self._rows_route(users[0]) is None or id(users[0]) in replace:
                continue
            g, u = ins[0], ins[2]
            shape = tuple(st.out.shape)
            if (tuple(g.shape) != shape or tuple(u.shape) != shape or not g.is_contiguous()
                    or not u.is_contiguous() or g.dtype != np.float32 or u.dtype != np.float32):
                continue
            mat = users[0]
            sh = self._rows_route(mat)
            replace[id(mat)] = rows_step(g, [mat], [(sh[0], sh[1], sh[2], g.shape[-1], sh[4])], [mat.out],
                                         x_mode=_lib.ROWS_X_SWIGLU, x2=u)
            removed.add(id(st))
        for st in steps:  # residual epilogues
            if st.name != "elementwise" or id(st) in removed:
                continue
            ins, ops = st.args["inputs"], st.args["instrs"]
            if len(ins) != 2 or [tuple(o[:3]) for o in ops] != [("add", 0, 1)] or np.dtype(ops[0][3]) != np.float32:
                continue
            shape = tuple(st.out.shape)
            for mi, ri in ((1, 0), (0, 1)):
                mv, r = ins[mi], ins[ri]
                mat = producer.get(id(mv.buf))
                if mat is None or id(mat) in removed:
                    continue
                cur = replace.get(id(mat), mat)
                users = readers.get(id(mv.buf), [])
                if (len(users) != 1 or id(mv.buf) in external or mv.offset != 0 or not mv.is_contiguous()
                        or tuple(mv.shape) != shape):
                    continue
                if cur.name == "matmul":
                    sh = self._rows_route(cur)
                    if sh is None:
                        continue
                    cur = rows_step(cur.args["a"], [cur], [sh], [cur.out])
                elif cur.name != "matmul_rows" or len(cur.args["weights"]) != 1 or cur.args["residual"] is not None:
                    continue
                if r.dtype != np.float32 or tuple(r.shape) != shape or not r.is_contiguous():
                    continue
                made = producer.get(id(r.buf))
                if made is not None and index[id(made)] > index[id(mat)]:
                    continue
                cur.args["residual"] = r
                cur.args["outs"] = [st.out]
                cur.out = st.out
                cur.text = cur.text[:-1] + ", epilogue=residual)"
                replace[id(mat)] = cur
                removed.add(id(st))
                break
        for st in steps:  # the rest: plain row GEMMs (an O projection feeding an all-reduce, or a bf16 residual)
            if id(st) in removed or id(st) in replace:
                continue
            sh = self._rows_route(st)
            if sh is not None:
                replace[id(st)] = rows_step(st.args["a"], [st], [sh], [st.out])
        plan.steps = [replace.get(id(st), st) for st in steps if id(st) not in removed]
        self._fuse_batched_attention()

    def _fuse_batched_attention(self) -> None:
        """RoPE(q), RoPE(k), the two cache blends and the attention of a batched decode step => one kernel.

        The chain of LlamaDecoderStep (llama.py:509-525) over B sequences at
        one position: q and k roped at ``position``, the write-mask blend
        ``cache*(1-wm) + row*wm`` of k and v into the caches (in place), then
        single-query attention.  When q, k and v are the three outputs of one
        row GEMM read by nothing else, that GEMM writes them as one
        (B, q | k | v) buffer and cb_decode_attention_batched runs the chain
        per (context split, KV head, sequence) -- the single-sequence decode
        attention's arithmetic, rebased per sequence.
        """
        plan = self.plan
        steps = plan.steps
        readers: Dict[int, List[Step]] = {}
        for st in steps:
            for b in _step_reads(st):
                readers.setdefault(b, []).append(st)
        external = {id(v.buf) for _, v in plan.outputs} | {id(b) for b in plan.argmax_of.values()}
        writer: Dict[int, Step] = {}
        for st in steps:
            if st.out is not None:
                writer[id(st.out.buf)] = st  # the last writer (kv_write updates caches in place)
        removed: Set[int] = set()
        replace: Dict[int, Step] = {}

        def only(view: View, reader: Step) -> bool:
            return (id(view.buf) not in external and readers.get(id(view.buf), []) == [reader])

        for st in steps:
            if st.name != "sdpa" or id(st) in removed:
                continue
            q, k, v, mask = (st.args[n] for n in ("q", "k", "v", "mask"))
            if len(q.shape) != 4 or q.shape[2] != 1 or len(k.shape) != 4:
                continue
            b, heads, _, hd = q.shape
            _, kvh, ctx, _ = k.shape
            if hd not in (32, 64, 128, 256) or heads % kvh or tuple(v.shape) != tuple(k.shape):
                continue
            if tuple(mask.shape) != (1, 1, 1, ctx) or not mask.is_contiguous() or not st.out.is_contiguous():
                continue
            rq = writer.get(id(q.buf))
            kwk, kwv = writer.get(id(k.buf)), writer.get(id(v.buf))
            if (rq is None or kwk is None or kwv is None or rq.name != "rope" or kwk.name != "kv_write"
                    or kwv.name != "kv_write" or rq.out is not q and rq.out.buf is not q.buf):
                continue
            rk = writer.get(id(kwk.args["row"].buf))
            if rk is None or rk.name != "rope" or not only(q, st) or not only(rk.out, kwk):
                continue
            if (kwk.args["write_mask"].buf is not kwv.args["write_mask"].buf
                    or np.dtype(kwk.args["one_minus"]) != np.dtype(kwv.args["one_minus"])
                    or rq.args["offset"] is None or rk.args["offset"] is None
                    or rq.args["offset"].buf is not rk.args["offset"].buf
                    or not _same_table(rq.args["cos"], rk.args["cos"])
                    or not _same_table(rq.args["sin"], rk.args["sin"])):
                continue
            xq, xk, xv = rq.args["x"], rk.args["x"], kwv.args["row"]
            m = writer.get(id(xq.buf))
            if m is None or m.name != "matmul_rows" or len(m.args["outs"]) != 3 or id(m) in replace:
                continue
            outs = m.args["outs"]
            if not (xq.buf is outs[0].buf and xk.buf is outs[1].buf and xv.buf is outs[2].buf):
                continue
            if not (only(xq, rq) and only(xk, rk) and only(xv, kwv)):
                continue
            nq, nk = heads * hd, kvh * hd
            if tuple(outs[0].shape[-1:]) != (nq,) or outs[1].shape[-1] != nk or outs[2].shape[-1] != nk:
                continue
            if any(o.size != b * o.shape[-1] for o in outs) or m.args["m"] != b:
                continue
            row = nq + 2 * nk
            qkv = self.plan.buffer("tmp", (b, row), F32)
            cols = (0, nq, nq + nk)
            m.args["outs"] = [View(qkv, (b, 1, n), (row, n, 1), c) for n, c in zip((nq, nk, nk), cols)]
            m.args["ldo"] = [row, row, row]
            m.out = m.args["outs"][0]
            splits = -(-ctx // 32)
            scratch = self.aux(shape=(b * splits * heads * (hd + 2),), dtype=np.float32)
            counters = self.aux(shape=(b * kvh,), dtype=np.int32, zero=True)  # used as unsigned
            kc, vc = kwk.args["cache"], kwv.args["cache"]
            fused = Step("decode_attention_batched", st.out, dict(
                qkv=View.whole(qkv), q_off=0, k_off=nq, v_off=nq + nk, batch=b, qkv_stride=row,
                heads=heads, kv_heads=kvh, head_size=hd, context=ctx, position=rq.args["offset"],
                cos=rq.args["cos"], sin=rq.args["sin"], n_positions=rq.args["n_offsets"],
                k_cache=kc, v_cache=vc, write_mask=kwk.args["write_mask"], one_minus=kwk.args["one_minus"],
                mask=mask, divisor=st.args["divisor"], scratch=scratch, counters=counters, flag=self.error_flag()),
                f"decode_attention_batched(qkv={qkv.name}, kv=({self._name(kc)}, {self._name(vc)}), batch={b})")
            replace[id(st)] = fused
            removed.update(id(x) for x in (rq, rk, kwk, kwv))
        plan.steps = [replace.get(id(st), st) for st in steps if id(st) not in removed]
        for st in plan.steps:
            if st.name == "kv_write" and st.args["cache"].dtype != F32:
                raise PlanError("a bfloat16 KV cache is updated only by the fused decode attention kernels "
                                "(bfloat16 weights on the tensor-core row GEMM); this graph needs float32 caches")

    PURE_STEPS = frozenset(("elementwise", "matmul", "reduce", "copy", "rms_norm", "rope", "sdpa", "place"))

    def _drop_dead_steps(self) -> None:
        """Remove pure steps whose output no later step or program output reads.

        Sub-expressions absorbed into a fused elementwise group can also be
        emitted on their own (a lowering or a second path referenced them);
        when nothing reads that copy it is dead work.  Temporary buffers left
        without a writer are dropped too.
        """
        plan = self.plan
        live = {id(v.buf) for _, v in plan.outputs}
        live.update(id(b) for b in plan.argmax_of.values())
        kept: List[Step] = []
        for step in reversed(plan.steps):
            if step.name in self.PURE_STEPS and step.out is not None and id(step.out.buf) not in live:
                continue
            kept.append(step)
            _collect_buffers(step.args, live)
            if step.out is not None:
                live.add(id(step.out.buf))
        plan.steps = kept[::-1]
        for init in plan.init_steps:
            _collect_buffers(init, live)
        plan.buffers = [b for b in plan.buffers if b.kind != "tmp" or id(b) in live]

    def _pruned_leaves(self) -> Set[object]:
        """Leaves only reachable through portable sub-graphs of used lowerings."""
        seen, stack = set(), list(self.outputs)
        while stack:
            n = stack.pop()
            if n in seen:
                continue
            seen.add(n)
            stack.extend(n.inputs)
        return {n for n in seen if n.op is None}

    def _bind_leaf(self, leaf) -> None:
        dt = self.rdt(leaf)
        dynamic = leaf in self.dynamic
        cached = (not dynamic) and leaf.cache_native
        buf = self.plan.buffer("input", leaf.shape, dt, node=leaf,
                               bind="pointer" if cached else "copy")
        self.plan.input_buffers[leaf] = buf
        self._val[leaf] = View.whole(buf)

    def value(self, node) -> View:
        if node not in self._val:
            self._emit_generic(node)
        return self._val[node]

    def set_value(self, node, view: View) -> None:
        self._val[node] = view

    def tmp(self, shape, dtype) -> View:
        return View.whole(self.plan.buffer("tmp", shape, dtype))

    def aux(self, host: Optional[np.ndarray] = None, *, shape=None, dtype=None, zero=False) -> Buffer:
        if host is not None:
            return self.plan.buffer("aux", host.shape, host.dtype, host=host)
        return self.plan.buffer("aux", shape, dtype, zero=zero)

    def error_flag(self) -> Buffer:
        if self.plan.error_flag is None:
            self.plan.error_flag = self.aux(shape=(1,), dtype=np.int32, zero=True)
        return self.plan.error_flag

    def add_step(self, name: str, out: Optional[View], text: str, **args) -> Step:
        step = Step(name, out, args, text)
        self.plan.steps.append(step)
        return step

    def contiguous(self, view: View) -> View:
        if view.is_contiguous():
            return view
        out = self.tmp(view.shape, view.dtype)
        self.add_step("copy", out, f"copy({self._name(view)})", src=view)
        return out

    def _name(self, view: View) -> str:
        return view.buf.name + (f"[+{view.offset}]" if view.offset else "")

    # ------------------------------------------------- generic emission
    def _emit_generic(self, node) -> None:
        if node in self._val:
            return
        # make sure parents exist first (iterative to avoid deep recursion)
        pending = [node]
        while pending:
            top = pending[-1]
            missing = [p for p in self._parents(top) if p not in self._val]
            if missing:
                pending.extend(missing)
                continue
            pending.pop()
            if top not in self._val:
                self._emit_one(top)

    def _emit_one(self, node) -> None:
        low = self._low.get(node)
        if low is not None:
            getattr(self, f"_emit_{low[0]}")(node, low)
            return
        k = kind(node)
        getattr(self, f"_emit_{k}")(node)

    def _emit_reshape(self, node) -> None:
        src = self.value(node.inputs[0])
        strides = reshape_strides(src.shape, src.strides, node.arg)
        if strides is None:
            src = self.contiguous(src)
            strides = contiguous_strides(node.arg)
        self.set_value(node, View(src.buf, tuple(node.arg), strides, src.offset))

    def _emit_permute(self, node) -> None:
        src = self.value(node.inputs[0])
        axes = tuple(node.arg)
        self.set_value(node, View(src.buf, tuple(src.shape[a] for a in axes),
                                  tuple(src.strides[a] for a in axes), src.offset))

    def _emit_elementwise(self, node) -> None:
        group = self._ew_groups.get(node)
        if group is None:
            group = self._ew_tree(node, set())
        inputs, instrs = group
        views = [self.value(p) for p in inputs]
        out = self.tmp(node.shape, self.rdt(node))
        self.add_step("elementwise", out,
                      f"elementwise({', '.join(self._name(v) for v in views)}; "
                      f"{' '.join(i[0] for i in instrs)})",
                      inputs=views, instrs=instrs, shape=tuple(node.shape))
        self.set_value(node, out)

    def _ew_tree(self, root, absorbed: Set[object]):
        inputs: List[object] = []
        slot: Dict[object, int] = {}
        instrs: List[Tuple[str, int, int, np.dtype]] = []
        reg: Dict[object, int] = {}

        order: List[object] = []
        stack = [(root, False)]
        while stack:
            n, done = stack.pop()
            if done:
                order.append(n)
                continue
            if n in reg:
                continue
            if n is root or n in absorbed:
                stack.append((n, True))
                for p in reversed(n.inputs):
                    stack.append((p, False))
        for n in order:
            if n in reg:
                continue
            operands = []
            for p in n.inputs:
                if p is root or p in absorbed:
                    operands.append(("r", p))
                else:
                    if p not in slot:
                        slot[p] = len(inputs)
                        inputs.append(p)
                    operands.append(("i", p))
            reg[n] = len(instrs)
            instrs.append((str(n.arg), operands, self.rdt(n)))
        n_in = len(inputs)
        encoded = []
        for name, operands, dt in instrs:
            idx = []
            for tag, p in operands:
                idx.append(slot[p] if tag == "i" else n_in + reg[p])
            encoded.append((name, idx[0], idx[1] if len(idx) > 1 else -1, dt))
        return inputs, encoded

    def _fuse_elementwise_groups(self) -> None:
        """Inline single-consumer elementwise parents of the same shape."""
        self._ew_groups: Dict[object, tuple] = {}
        candidates = [n for n in self.order
                      if is_ew(n) and n not in self._low and n not in self._val
                      and n not in self.claimed and n not in self.units]
        cand = set(candidates)
        absorbed: Set[object] = set()
        for child in candidates:
            for p in child.inputs:
                if (p in cand and p.shape == child.shape and p not in self.output_set
                        and len(self.consumers.get(p, ())) == 1):
                    absorbed.add(p)
        for root in candidates:
            if root in absorbed:
                continue
            mine = set()
            stack = [root]
            while stack:
                n = stack.pop()
                for p in n.inputs:
                    if p in absorbed and p not in mine:
                        mine.add(p)
                        stack.append(p)
            inputs, instrs = self._ew_tree(root, mine)
            while len(inputs) > _lib.EW_MAX_INPUTS or len(instrs) > _lib.EW_MAX_INSTR:
                # too big: stop absorbing the root's direct parents
                for p in root.inputs:
                    mine.discard(p)
                    absorbed.discard(p)
                inputs, instrs = self._ew_tree(root, mine)
                if len(inputs) > _lib.EW_MAX_INPUTS:
                    raise PlanError("elementwise node with too many operands")
            self._ew_groups[root] = (inputs, instrs)
        for n in absorbed:
            self.claimed.add(n)

    def _emit_reduce(self, node) -> None:
        src = self.value(node.inputs[0])
        how, axes, keepdims = node.arg
        axes = tuple(axes)
        keep = [d for d in range(len(src.shape)) if d not in axes]
        dt = self.rdt(node)
        out = self.tmp(node.shape, dt)
        sequential = how == "sum" and dt.name in ("bfloat16", "float16")
        self.add_step("reduce", out, f"reduce_{how}({self._name(src)}, axis={axes})",
                      src=src, how=how, keep=keep, red=list(axes), sequential=sequential)
        self.set_value(node, out)

    def _placement_columns(self, node) -> Optional[np.ndarray]:
        """Source row of each column when the right operand is a placement matrix.

        The prefill's KV-cache placement (llama.py:243-247, used at 411-418)
        is a constant 0/1 matrix with one 1 per row and at most one per
        column; ``x @ P`` then copies columns of x (products by 1, sums with
        zeros: exact).  Returns int32 sources (-1 = zero column) or None.
        """
        p = node.inputs[1]
        if p.op is not None or p in self.dynamic or len(p.shape) != 2 or len(node.inputs[0].shape) < 1:
            return None
        if p.shape[0] * p.shape[1] > (1 << 26) or p.shape[0] >= (1 << 31):
            return None
        try:
            value = np.asarray(p.numpy_value())
        except Exception:
            return None
        ones = value == 1
        if not np.all(ones | (value == 0)):
            return None
        if np.any(ones.sum(axis=1) != 1) or np.any(ones.sum(axis=0) > 1):
            return None
        cols = np.full(p.shape[1], -1, dtype=np.int32)
        rows, where = np.nonzero(ones)
        cols[where] = rows
        if not p.cache_native:
            self.plan.guards.append((p, value.copy()))
        return cols

    def _emit_matmul(self, node) -> None:
        cols = self._placement_columns(node)
        if cols is not None:
            a = self.value(node.inputs[0])
            dt = self.rdt(node)
            out = self.tmp(node.shape, bf16() if self.kv_bf16 and dt == F32 else dt)
            self.plan.lowered["place"] = self.plan.lowered.get("place", 0) + 1
            table = self.aux(cols)
            self.add_step("place", out, f"place({self._name(a)}, cols={table.name})", src=a, cols=table)
            self.set_value(node, out)
            return
        a, b = (self.value(p) for p in node.inputs)
        out = self.tmp(node.shape, self.rdt(node))
        self.add_step("matmul", out, f"matmul({self._name(a)}, {self._name(b)})", a=a, b=b)
        self.set_value(node, out)

    def _emit_gather(self, node) -> None:
        table = self.contiguous(self.value(node.inputs[0]))
        idx = self.contiguous(self.value(node.inputs[1]))
        if np.dtype(idx.dtype).name not in ("int32", "int64"):
            raise PlanError("gather indices must be int32 or int64 on cuda-b200")
        out = self.tmp(node.shape, self.rdt(node))
        self.add_step("gather", out, f"gather({self._name(table)}, {self._name(idx)})",
                      table=table, idx=idx, flag=self.error_flag())
        self.set_value(node, out)

    # lowerings --------------------------------------------------------
    def _emit_rms_norm(self, node, low) -> None:
        x, w = (self.contiguous(self.value(p)) for p in low[1])
        spec = self._rms[node]
        out = self.tmp(node.shape, spec.out_dtype)
        self.plan.lowered["rms_norm"] = self.plan.lowered.get("rms_norm", 0) + 1
        self.add_step("rms_norm", out, f"rms_norm({self._name(x)}, {self._name(w)}, "
                      f"eps={spec.eps!r}, divisor={spec.divisor!r})", x=x, w=w, spec=spec)
        self.set_value(node, out)

    def rope_tables(self, node) -> Tuple[Buffer, Buffer, int]:
        info = self._rope[node]
        if info[0] == "table":
            _, cos, sin = info
            return self.aux(cos), self.aux(sin), 1
        _, theta, dtype, tokens, hd = info
        key = ("rope", theta, np.dtype(dtype).str, tokens, hd, self.max_positions)
        cached = self.table_cache.get(key)
        if cached is None:
            from .graphs import rope_angles

            angles = rope_angles(self.max_positions + tokens - 1, hd, theta)
            cos = np.cos(angles).astype(dtype).astype(np.float32)
            sin = np.sin(angles).astype(dtype).astype(np.float32)
            # row p of offset o is angle o + p: [n_offsets][T][half]
            idx = np.arange(self.max_positions)[:, None] + np.arange(tokens)[None, :]
            cached = (cos[idx].copy(), sin[idx].copy())
            self.table_cache[key] = cached
        return self.aux(cached[0]), self.aux(cached[1]), self.max_positions

    def _emit_rope(self, node, low) -> None:
        x = self.value(low[1][0])
        cos, sin, n_off = self.rope_tables(node)
        offset = self.contiguous(self.value(low[1][1])) if len(low[1]) == 2 else None
        out = self.tmp(node.shape, self.rdt(node))
        self.plan.lowered["rope"] = self.plan.lowered.get("rope", 0) + 1
        self.add_step("rope", out, f"rope({self._name(x)}, theta={low[2][1]!r})", x=x, cos=cos,
                      sin=sin, n_offsets=n_off, offset=offset, flag=self.error_flag())
        self.set_value(node, out)

    def _causal_mask(self, mask) -> int:
        """cb_sdpa_tc causal flags a constant mask allows (0 = none).

        CB_CAUSAL_SKIP when the mask is <= -5000 at every key past the causal
        diagonal j > i + (tk - tq): those keys add exp(...) == 0 exactly and
        key tiles made only of them are skipped.  CB_CAUSAL_ZERO_BELOW as well
        when it is exactly 0 at every other key (then it is read only on the
        diagonal tiles).  The prefill's mask (llama.py:250-258: -1e4 above
        the diagonal, 0 elsewhere) has both.
        """
        if mask.op is not None or mask in self.dynamic or len(mask.shape) < 2:
            return 0
        tq, tk = mask.shape[-2:]
        if int(np.prod(mask.shape)) > (1 << 26) or tk < tq:
            return 0
        try:
            value = np.asarray(mask.numpy_value()).astype(np.float32).reshape(-1, tq, tk)
        except Exception:
            return 0
        above = np.arange(tk)[None, :] > np.arange(tq)[:, None] + (tk - tq)
        if not np.all(value[:, above] <= -5000.0):
            return 0
        if not mask.cache_native:
            self.plan.guards.append((mask, np.asarray(mask.numpy_value()).copy()))
        flags = _lib.CAUSAL_SKIP
        if np.all(value[:, ~above] == 0.0):
            flags |= _lib.CAUSAL_ZERO_BELOW
        return flags

    # ------------------------------------------------------------ training
    def _rows_view(self, node):
        v = self.contiguous(self.value(node))
        width = v.shape[-1] if v.shape else 1
        return v, (v.size // width if width else 0), width

    def _emit_softmax(self, node, low, log_form: bool = False, name: str = "softmax") -> None:
        x, rows, width = self._rows_view(low[1][0])
        out = self.tmp(node.shape, F32)
        self.plan.lowered[name] = self.plan.lowered.get(name, 0) + 1
        self.add_step("softmax", out, f"{name}({self._name(x)}, axis=-1)", x=x, rows=rows, width=width,
                      log=log_form)
        self.set_value(node, out)

    def _emit_log_softmax(self, node, low) -> None:
        self._emit_softmax(node, low, True, "log_softmax")

    def _emit_softmax_backward(self, node, low, log_form: bool = False, name: str = "softmax_backward") -> None:
        g, rows, width = self._rows_view(low[1][0])
        y = self.contiguous(self.value(low[1][1]))
        out = self.tmp(node.shape, F32)
        self.plan.lowered[name] = self.plan.lowered.get(name, 0) + 1
        self.add_step("softmax_backward", out, f"{name}({self._name(g)}, {self._name(y)}, axis=-1)", grad=g, y=y,
                      rows=rows, width=width, log=log_form)
        self.set_value(node, out)

    def _emit_log_softmax_backward(self, node, low) -> None:
        self._emit_softmax_backward(node, low, True, "log_softmax_backward")

    def _emit_layer_norm(self, node, low) -> None:
        x, rows, width = self._rows_view(low[1][0])
        w, b = (self.contiguous(self.value(n)) for n in low[1][1:])
        out = self.tmp(node.shape, F32)
        eps = float(np.float32(low[2]))
        self.plan.lowered["layer_norm"] = self.plan.lowered.get("layer_norm", 0) + 1
        self.add_step("layer_norm", out, f"layer_norm({self._name(x)}, {self._name(w)}, {self._name(b)}, "
                      f"eps={eps!r})", x=x, w=w, b=b, rows=rows, width=width, eps=eps)
        self.set_value(node, out)

    def _emit_layer_norm_backward(self, node, low) -> None:
        """One step for every requested contribution (input, weight, bias) of the same backward."""
        inputs, eps = low[1], float(np.float32(low[2][0]))
        siblings = {}
        for other in self.order:
            olow = self._low.get(other)
            if (olow is not None and olow[0] == "layer_norm_backward" and tuple(olow[1]) == tuple(inputs)
                    and float(np.float32(olow[2][0])) == eps and other not in self._val):
                siblings.setdefault(olow[2][1], other)
        siblings.setdefault(low[2][1], node)
        g, rows, width = self._rows_view(inputs[0])
        x = self.contiguous(self.value(inputs[1]))
        w = self.contiguous(self.value(inputs[2]))
        outs = {which: self.tmp(n.shape, F32) for which, n in siblings.items()}
        stats = self.aux(shape=(max(rows, 1) * 2,), dtype=np.float32) if 1 in outs else None
        names = ", ".join(self._name(outs[k]) if k in outs else "_" for k in (0, 1, 2))
        self.plan.lowered["layer_norm_backward"] = self.plan.lowered.get("layer_norm_backward", 0) + 1
        self.add_step("layer_norm_backward", outs[min(outs)],
                      f"layer_norm_backward({self._name(g)}, {self._name(x)}, {self._name(w)}, eps={eps!r})"
                      f" -> ({names})", grad=g, x=x, w=w, rows=rows, width=width, eps=eps,
                      dx=outs.get(0), dw=outs.get(1), db=outs.get(2), stats=stats)
        for which, n in siblings.items():
            self.set_value(n, outs[which])

    def _emit_all_reduce(self, node, low) -> None:
        src = self.contiguous(self.value(low[1][0]))
        out = self.tmp(node.shape, src.dtype)
        self.plan.lowered["all_reduce"] = self.plan.lowered.get("all_reduce", 0) + 1
        self.add_step("all_reduce", out, f"all_reduce({self._name(src)}, group={low[2]!r})", src=src,
                      group=low[2], flag=self.error_flag())  # the peer kernel reports a rank that did not arrive
        self.set_value(node, out)

    def _emit_all_gather(self, node, low) -> None:
        src = self.contiguous(self.value(low[1][0]))
        out = self.tmp(node.shape, src.dtype)
        self.plan.lowered["all_gather"] = self.plan.lowered.get("all_gather", 0) + 1
        self.add_step("all_gather", out, f"all_gather({self._name(src)}, group={low[2]!r})", src=src,
                      group=low[2])
        self.set_value(node, out)

    def _emit_sdpa(self, node, low) -> None:
        q, k, v, mask = (self.value(p) for p in low[1])
        b, h, t, d = node.shape
        users = self.consumers.get(node, [])
        if (t > 1 and len(users) == 1 and kind(users[0]) == "permute" and tuple(users[0].arg) == (0, 2, 1, 3)
                and node not in self.output_set):
            # the graph merges the heads next (llama.py:362-363): write token-major
            # rows, so the permute is a view and the merge needs no copy
            buf = self.plan.buffer("tmp", (b, t, h, d), F32)
            out = View(buf, (b, h, t, d), (t * h * d, d, h * d, 1), 0)
        else:
            out = self.tmp(node.shape, F32)
        causal = self._causal_mask(low[1][3])
        self.plan.lowered["sdpa"] = self.plan.lowered.get("sdpa", 0) + 1
        self.add_step("sdpa", out, f"sdpa({self._name(q)}, {self._name(k)}, {self._name(v)}, "
                      f"mask={self._name(mask)}, divisor={self._sdpa[node]!r}"
                      f"{', causal=%d' % causal if causal else ''})",
                      q=q, k=k, v=v, mask=mask, divisor=self._sdpa[node], causal=causal)
        self.set_value(node, out)

    # ------------------------------------------------------------ source
    def _source(self) -> str:
        lines = ["def run(inputs):"]
        for buf in self.plan.buffers:
            if buf.kind == "input":
                lines.append(f"    {buf.name} = input({buf.bind}) {buf.shape} {buf.dtype}")
        for step in self.plan.steps:
            target = self._name(step.out) if step.out is not None else "_"
            lines.append(f"    {target} = {step.text}")
        outs = ", ".join(self._name(v) + (" (in place)" if i in self.plan.aliases else "")
                         for i, (_, v) in enumerate(self.plan.outputs))
        lines.append(f"    return ({outs},)")
        return "\n".join(lines)
