"""Host-side mirror of chomik-grad's six-operation IR and plugin contract.

This module restates the public interface of ``chomikgrad/lazy.py`` so that
the ``cuda-b200`` plugin and the Llama graph builders run on machines where the
reference package is not installed.  Names, argument meaning and error
behaviour follow the reference:

* ``Op`` (six instructions)                      -- lazy.py:22-34
* ``LazyNode`` (+ ``leaf``/``native_leaf``/``numpy_value``) -- lazy.py:37-104
* ``DeviceAdapter`` / ``CompiledProgram`` / ``Compiler`` ABCs -- lazy.py:107-209
* ``topological_sort``                           -- lazy.py:212-233
* ``GraphPlan`` (lowering overrides, signature, elementwise fusion plan)
                                                 -- lazy.py:236-378
* ``register_compiler`` / ``set_default_compiler`` / ``get_compiler``
                                                 -- lazy.py:646-678

The compiler in :mod:`cuda_b200.compiler` never relies on these classes by
identity: it reads nodes through their attributes (``op.value``, ``inputs``,
``arg``, ``shape``, ``dtype``, ``lowering`` ...), so graphs built by the real
``chomikgrad`` package compile the same way (see :func:`cuda_b200.install`).

No compute lives here.  There is deliberately no NumPy compiler in the
product: the ``cpu`` compiler is the parity oracle and is registered by the
test-only ``oracle`` package.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from enum import Enum
from pathlib import Path
from typing import (
    Callable,
    Dict,
    Iterable,
    Mapping,
    Optional,
    Sequence,
    Tuple,
    Union,
)

import numpy as np


class Op(Enum):
    """The six graph instructions (lazy.py:22-34).

    Elementwise variants (add, exp, ...) are the ``arg`` of ELEMENTWISE.
    """

    ELEMENTWISE = "elementwise"
    REDUCE = "reduce"
    RESHAPE = "reshape"
    PERMUTE = "permute"
    MATMUL = "matmul"
    GATHER = "gather"


Lowering = Tuple[str, Tuple["LazyNode", ...], object]


class LazyNode:
    """One graph value (lazy.py:37-104).

    ``native_values`` maps a backend name to device storage; leaves without a
    host ``value`` are read back through that backend's device adapter.
    """

    __slots__ = (
        "op",
        "inputs",
        "arg",
        "shape",
        "dtype",
        "value",
        "native_values",
        "cache_native",
        "lowering",
    )

    def __init__(
        self,
        op: Optional[Op],
        inputs: Sequence["LazyNode"],
        arg: object,
        shape: Tuple[int, ...],
        dtype: np.dtype,
        value: Optional[np.ndarray] = None,
        native_values: Optional[Dict[str, object]] = None,
        cache_native: bool = True,
        lowering: Optional[Lowering] = None,
    ) -> None:
        self.op = op
        self.inputs = tuple(inputs)
        self.arg = arg
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.value = value
        self.native_values = native_values if native_values else {}
        self.cache_native = cache_native
        self.lowering = lowering

    @classmethod
    def leaf(cls, value: np.ndarray, *, cache_native: bool = True) -> "LazyNode":
        return cls(None, (), None, value.shape, value.dtype, value,
                   cache_native=cache_native)

    @classmethod
    def native_leaf(
        cls,
        backend: str,
        value: object,
        shape: Tuple[int, ...],
        dtype: np.dtype,
    ) -> "LazyNode":
        return cls(None, (), None, shape, dtype, native_values={backend: value})

    def numpy_value(self) -> np.ndarray:
        """Host value of a leaf; native-only leaves are read back once."""
        if self.value is not None:
            return self.value
        if not self.native_values:
            raise RuntimeError("leaf node has no value")
        backend, native = next(iter(self.native_values.items()))
        try:
            host = get_compiler(backend).device.to_numpy(native)
        except KeyError:
            host = native
        self.value = np.array(host, copy=True)
        return self.value


class DeviceAdapter(ABC):
    """Runtime boundary of a compiled device backend (lazy.py:107-151)."""

    name: str

    @abstractmethod
    def array(self, value: object) -> object:
        raise NotImplementedError

    @abstractmethod
    def evaluate(self, values: Sequence[object]) -> None:
        raise NotImplementedError

    @abstractmethod
    def synchronize(self) -> None:
        raise NotImplementedError

    @abstractmethod
    def to_numpy(self, value: object) -> np.ndarray:
        raise NotImplementedError

    @abstractmethod
    def argmax(self, value: object) -> int:
        raise NotImplementedError

    def argmax_last_axis(self, value: object) -> np.ndarray:
        return np.asarray(self.to_numpy(value)).argmax(axis=-1)

    @abstractmethod
    def dtype(self, value: object) -> np.dtype:
        raise NotImplementedError

    def load_safetensors(
        self, path: Path, *, dtype: Optional[np.dtype] = None
    ) -> Mapping[str, object]:
        raise NotImplementedError(
            f"the {self.name!r} device does not support safetensors loading"
        )

    def reset_peak_memory(self) -> None:
        pass

    def peak_memory_bytes(self) -> Optional[int]:
        return None


class CompiledProgram(ABC):
    """An executable program (lazy.py:154-169)."""

    source: str
    device: DeviceAdapter

    @abstractmethod
    def run(
        self,
        bindings: Optional[Mapping[LazyNode, object]] = None,
        *,
        synchronize: bool = False,
    ) -> Tuple[object, ...]:
        raise NotImplementedError

    def __call__(self) -> Tuple[np.ndarray, ...]:
        produced = self.run(synchronize=True)
        return tuple(self.device.to_numpy(item) for item in produced)


class Compiler(ABC):
    """A plugin turning lazy nodes into a program (lazy.py:172-209)."""

    device: DeviceAdapter

    @abstractmethod
    def compile(
        self,
        outputs: Sequence[LazyNode],
        dynamic_inputs: Sequence[LazyNode] = (),
    ) -> CompiledProgram:
        raise NotImplementedError

    def update_parameters(
        self,
        parameters: Sequence[LazyNode],
        gradients: Sequence[LazyNode],
        learning_rate: float,
        *,
        inplace: bool = False,
    ) -> Optional[Tuple[Tuple[LazyNode, ...], Tuple[LazyNode, ...]]]:
        if inplace:
            raise RuntimeError(
                "this compiler does not support in-place parameter updates"
            )
        return None

    def update_native_parameters(
        self,
        parameters: Sequence[LazyNode],
        gradients: Sequence[object],
        learning_rate: float,
        *,
        inplace: bool = False,
    ) -> Tuple[Tuple[LazyNode, ...], Tuple[LazyNode, ...]]:
        raise RuntimeError("this compiler does not support compiled training steps")


def _walk(outputs: Iterable[LazyNode],
          parents_of: Callable[[LazyNode], Sequence[LazyNode]]) -> Tuple[LazyNode, ...]:
    """Post-order DFS shared by the sorters below.

    Iterative (graphs of a 32-layer model are thousands of nodes deep), but it
    visits parents in the same order as the recursive reference walk, so the
    node order -- and therefore ``GraphPlan.signature`` -- is identical.
    """
    order = []
    seen = set()
    for root in outputs:
        if root in seen:
            continue
        seen.add(root)
        stack = [(root, iter(parents_of(root)))]
        while stack:
            node, pending = stack[-1]
            advanced = False
            for parent in pending:
                if parent not in seen:
                    seen.add(parent)
                    stack.append((parent, iter(parents_of(parent))))
                    advanced = True
                    break
            if not advanced:
                stack.pop()
                order.append(node)
    return tuple(order)


def topological_sort(
    outputs: Iterable[LazyNode], *, use_lowerings: bool = False
) -> Tuple[LazyNode, ...]:
    """Parents-first order (lazy.py:212-233)."""
    if use_lowerings:
        return _walk(outputs, lambda n: n.lowering[1] if n.lowering is not None
                     else n.inputs)
    return _walk(outputs, lambda n: n.inputs)


class GraphPlan:
    """Backend-local lowering choices over a shared graph (lazy.py:236-378).

    A backend chooses which intrinsic lowerings it honours; fusions are kept
    in ``_overrides`` so the portable graph itself is never mutated.
    """

    def __init__(self, outputs: Sequence[LazyNode],
                 supported_lowerings: Iterable[str]) -> None:
        if not outputs:
            raise ValueError("at least one output is required")
        self.outputs = tuple(outputs)
        self.supported_lowerings = frozenset(supported_lowerings)
        self._overrides: Dict[LazyNode, Lowering] = {}

    def lowering(self, node: LazyNode) -> Optional[Lowering]:
        chosen = self._overrides.get(node)
        if chosen is not None:
            return chosen
        intrinsic = node.lowering
        if intrinsic is not None and intrinsic[0] in self.supported_lowerings:
            return intrinsic
        return None

    def inputs(self, node: LazyNode) -> Tuple[LazyNode, ...]:
        chosen = self.lowering(node)
        return chosen[1] if chosen is not None else node.inputs

    def nodes(self) -> Tuple[LazyNode, ...]:
        return _walk(self.outputs, self.inputs)

    def signature(self, nodes: Optional[Sequence[LazyNode]] = None) -> object:
        """Structural key: equal for graphs that differ only in leaf values."""
        selected = tuple(nodes) if nodes is not None else self.nodes()
        position = {node: index for index, node in enumerate(selected)}
        entries = []
        for node in selected:
            chosen = self.lowering(node)
            if node.op is None:
                entries.append((None, node.shape, node.dtype.str))
            elif chosen is not None:
                kind, inputs, argument = chosen
                entries.append(("lowering", kind, argument, node.shape,
                                node.dtype.str,
                                tuple(position[p] for p in inputs)))
            else:
                entries.append((node.op.value, node.arg, node.shape,
                                node.dtype.str,
                                tuple(position[p] for p in node.inputs)))
        return tuple(entries), tuple(position[n] for n in self.outputs)

    def fuse_elementwise(self) -> None:
        """Record single-consumer float32 elementwise chains as one fusion."""
        nodes = self.nodes()
        uses: Dict[LazyNode, int] = {}
        for node in nodes:
            for parent in self.inputs(node):
                uses[parent] = uses.get(parent, 0) + 1
        outputs = set(self.outputs)
        f32 = np.dtype(np.float32)

        def fusable(node: LazyNode) -> bool:
            return (node.op is not None and node.op.value == "elementwise"
                    and node.lowering is None and node not in self._overrides
                    and node.dtype == f32)

        absorbed = set()
        for child in nodes:
            if not fusable(child):
                continue
            for parent in child.inputs:
                if (fusable(parent) and parent.shape == child.shape
                        and uses.get(parent) == 1 and parent not in outputs):
                    absorbed.add(parent)

        for root in nodes:
            if not fusable(root) or root in absorbed:
                continue
            operands = []
            slot: Dict[LazyNode, int] = {}
            fused = 0

            def tree(node: LazyNode) -> object:
                nonlocal fused
                if node is root or node in absorbed:
                    fused += 1
                    return (str(node.arg), *(tree(p) for p in node.inputs))
                if node not in slot:
                    slot[node] = len(operands)
                    operands.append(node)
                return ("input", slot[node])

            expression = tree(root)
            if fused > 1:
                self._overrides[root] = ("elementwise_fusion", tuple(operands),
                                         expression)


CompilerFactory = Callable[[], Compiler]
CompilerRegistration = Union[Compiler, CompilerFactory]
_REGISTRY: Dict[str, CompilerRegistration] = {}
_INSTANCES: Dict[str, Compiler] = {}
_DEFAULT = ["cuda-b200"]


def register_compiler(name: str, compiler: CompilerRegistration, *,
                      replace: bool = False) -> None:
    """Register a compiler instance or factory (lazy.py:646-656)."""
    if not name:
        raise ValueError("compiler name cannot be empty")
    if name in _REGISTRY and not replace:
        raise ValueError(f"compiler already registered: {name}")
    if not isinstance(compiler, Compiler) and not callable(compiler):
        raise TypeError("compiler must be a Compiler instance or a factory")
    _REGISTRY[name] = compiler
    _INSTANCES.pop(name, None)


def set_default_compiler(name: str) -> None:
    """Select the compiler used when none is named (lazy.py:659-663)."""
    if name not in _REGISTRY:
        raise KeyError(f"unknown compiler: {name}")
    _DEFAULT[0] = name


def get_compiler(name: Optional[str] = None) -> Compiler:
    """Instantiate (once) and return a registered compiler (lazy.py:666-678)."""
    chosen = name or _DEFAULT[0]
    if chosen in _INSTANCES:
        return _INSTANCES[chosen]
    try:
        registration = _REGISTRY[chosen]
    except KeyError as error:
        raise KeyError(f"unknown compiler: {chosen}") from error
    instance = registration() if callable(registration) else registration
    if not isinstance(instance, Compiler):
        raise TypeError(f"compiler factory {chosen!r} returned an invalid object")
    _INSTANCES[chosen] = instance
    return instance


def realize_nodes(outputs: Sequence[LazyNode],
                  compiler: Optional[str] = None) -> Tuple[np.ndarray, ...]:
    return get_compiler(compiler).compile(outputs)()
