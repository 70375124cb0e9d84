"""PARITY ORACLE -- test infrastructure, not product code.

A CPU restatement of chomik-grad's ``cpu`` compiler (``chomikgrad/lazy.py``
:502-636): every graph node becomes one NumPy call, executed in topological
order, so results carry exactly the reference's dtype behaviour (including
ml_dtypes bfloat16 semantics: bf16 elementwise ops round per op, ``np.sum`` on
bf16 accumulates sequentially in bf16, ``np.matmul`` of bf16 operands returns
float32).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module.  The ``cuda-b200`` product never calls it.

Op mapping (lazy.py:554-568 and :609-636):
  ELEMENTWISE add/sub/mul/div/equal, neg/exp/log/sqrt/relu/step
  REDUCE      np.sum / np.max(axis, keepdims)
  RESHAPE     np.reshape;  PERMUTE np.transpose;  MATMUL np.matmul
  GATHER      np.take(table, ids, axis=0)
"""

from __future__ import annotations

from typing import Callable, Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from chomikgrad.lazy import (
    CompiledProgram,
    Compiler,
    DeviceAdapter,
    LazyNode,
    register_compiler,
    topological_sort,
)


def _binary(kind: str) -> Callable[[np.ndarray, np.ndarray], np.ndarray]:
    if kind == "add":
        return np.add
    if kind == "sub":
        return np.subtract
    if kind == "mul":
        return np.multiply
    if kind == "div":
        return np.divide
    if kind == "equal":
        return lambda a, b: np.equal(a, b).astype(a.dtype, copy=False)
    raise KeyError(kind)


def _unary(kind: str) -> Callable[[np.ndarray], np.ndarray]:
    table = {
        "neg": np.negative,
        "exp": np.exp,
        "log": np.log,
        "sqrt": np.sqrt,
        "relu": lambda a: np.maximum(a, 0),
        "step": lambda a: np.greater(a, 0).astype(a.dtype, copy=False),
    }
    return table[kind]


def evaluate_node(node: LazyNode, args: Sequence[np.ndarray]) -> np.ndarray:
    """One reference NumPy call for ``node`` (lazy.py:609-636)."""
    kind = node.op.value
    if kind == "elementwise":
        name = str(node.arg)
        if len(args) == 2:
            try:
                return _binary(name)(args[0], args[1])
            except KeyError:
                pass
        elif len(args) == 1:
            try:
                return _unary(name)(args[0])
            except KeyError:
                pass
        raise ValueError(f"unsupported elementwise operation: {name}")
    if kind == "reduce":
        how, axes, keepdims = node.arg
        if how == "sum":
            return np.sum(args[0], axis=axes, keepdims=keepdims)
        if how == "max":
            return np.max(args[0], axis=axes, keepdims=keepdims)
        raise ValueError(f"unsupported reduction: {how}")
    if kind == "reshape":
        return np.reshape(args[0], node.arg)
    if kind == "permute":
        return np.transpose(args[0], axes=node.arg)
    if kind == "matmul":
        return np.matmul(args[0], args[1])
    if kind == "gather":
        return np.take(args[0], args[1], axis=0)
    raise ValueError(f"unsupported operation: {node.op}")


class NumpyDeviceAdapter(DeviceAdapter):
    """Host 'device' of the oracle (lazy.py:528-548)."""

    name = "cpu"

    def array(self, value: object) -> np.ndarray:
        return np.asarray(value)

    def evaluate(self, values: Sequence[object]) -> None:
        for value in values:
            np.asarray(value)

    def synchronize(self) -> None:
        pass

    def to_numpy(self, value: object) -> np.ndarray:
        return np.asarray(value)

    def argmax(self, value: object) -> int:
        return int(np.asarray(value).argmax())

    def sample(self, value: object, *, temperature: float, top_k: int, rng: np.random.Generator) -> int:
        """The reference's host sampler (generate_tinyllama.py:124-157) on the oracle's arrays."""
        from .sampling import sample_token

        return sample_token(np.asarray(value), temperature=temperature, top_k=top_k, rng=rng)

    def sample_rows(self, value: object, *, temperature: float, top_k: int,
                    rng: np.random.Generator) -> np.ndarray:
        from .sampling import sample_token

        rows = np.asarray(value)
        flat = rows.reshape(-1, rows.shape[-1])
        out = [sample_token(flat[i:i + 1], temperature=temperature, top_k=top_k, rng=rng)
               for i in range(flat.shape[0])]
        return np.asarray(out, dtype=np.int64).reshape(rows.shape[:-1])

    def dtype(self, value: object) -> np.dtype:
        return np.asarray(value).dtype


class NumpyProgram(CompiledProgram):
    """Straight-line evaluation; unbound leaves read their host value (lazy.py:502-525)."""

    def __init__(self, order: Tuple[LazyNode, ...], outputs: Tuple[LazyNode, ...],
                 device: NumpyDeviceAdapter) -> None:
        self._order = order
        self._outputs = outputs
        self.inputs = tuple(n for n in order if n.op is None)
        self.device = device
        lines = ["def run(inputs):"]
        names = {n: f"v{i}" for i, n in enumerate(order)}
        for n in order:
            lines.append(f"    {names[n]} = " + ("input" if n.op is None else n.op.value))
        self.source = "\n".join(lines)

    def run(self, bindings: Optional[Mapping[LazyNode, object]] = None, *,
            synchronize: bool = False) -> Tuple[object, ...]:
        given = bindings or {}
        values: Dict[LazyNode, np.ndarray] = {}
        for node in self._order:
            if node.op is None:
                values[node] = (np.asarray(given[node]) if node in given
                                else node.numpy_value())
            else:
                values[node] = evaluate_node(node, [values[p] for p in node.inputs])
        return tuple(np.asarray(values[n]) for n in self._outputs)


class NumpyCompiler(Compiler):
    """The reference ``cpu`` compiler restated (lazy.py:551-607)."""

    def __init__(self) -> None:
        self.device = NumpyDeviceAdapter()

    def compile(self, outputs: Sequence[LazyNode],
                dynamic_inputs: Sequence[LazyNode] = ()) -> NumpyProgram:
        if not outputs:
            raise ValueError("at least one output is required")
        return NumpyProgram(topological_sort(outputs), tuple(outputs), self.device)


def install() -> None:
    """Register the oracle as the ``cpu`` compiler of chomikgrad's registry (tests only).

    It replaces the reference's own ``NumpyCompiler`` under that name in the
    test process, so every ``compiler="cpu"`` graph runs on the restatement;
    ``tests/test_oracle.py`` checks the restatement against the reference's
    compiler on the same graphs and against the golden fixtures.
    """
    register_compiler("cpu", NumpyCompiler, replace=True)


install()
