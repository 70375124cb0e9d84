"""Inference subset of chomik-grad's ``Tensor`` front-end (``chomikgrad/tensor.py``).

Every method builds exactly the nodes the reference builds -- same op, same
``arg``, same operand order, same metadata dtype (``np.result_type`` of the
operands, tensor.py:210-214) and the same intrinsic ``lowering`` tuples
(softmax tensor.py:325-334) -- so a graph built here has the same
``GraphPlan.signature`` as the reference's.  That equality is checked by the
CPU test suite against the real package.

Autograd is outside the inference hot path this package accelerates:
``requires_grad`` is recorded but ``backward`` raises.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Iterator, Optional, Sequence, Tuple, Union

import numpy as np

from .lazy import CompiledProgram, LazyNode, Op, get_compiler

ArrayLike = Union[float, int, Sequence[float], np.ndarray]
Axis = Optional[Union[int, Sequence[int]]]

_GRAD = [True]


@contextmanager
def no_grad() -> Iterator[None]:
    """Disable gradient tracking inside the block (tensor.py:18-26)."""
    saved = _GRAD[0]
    _GRAD[0] = False
    try:
        yield
    finally:
        _GRAD[0] = saved


def _axes(axis: Axis, ndim: int) -> Tuple[int, ...]:
    """Normalise reduction axes like tensor.py:29-38."""
    if axis is None:
        return tuple(range(ndim))
    listed = (axis,) if isinstance(axis, int) else tuple(axis)
    fixed = tuple(a + ndim if a < 0 else a for a in listed)
    if any(a < 0 or a >= ndim for a in fixed):
        raise ValueError(f"axis {axis!r} is invalid for a {ndim}D tensor")
    if len(set(fixed)) != len(fixed):
        raise ValueError("reduction axes must be unique")
    return fixed


def _kept(shape: Tuple[int, ...], axes: Tuple[int, ...], keepdims: bool) -> Tuple[int, ...]:
    if keepdims:
        return tuple(1 if i in axes else n for i, n in enumerate(shape))
    return tuple(n for i, n in enumerate(shape) if i not in axes)


class Tensor:
    """A lazy value; operations append ``LazyNode``s to the graph."""

    def __init__(self, data: ArrayLike, *, requires_grad: bool = False,
                 dtype: Optional[np.dtype] = None, copy: bool = True) -> None:
        array = np.asarray(data, dtype=dtype)
        if requires_grad and not np.issubdtype(array.dtype, np.floating):
            raise TypeError("only floating-point tensors can require gradients")
        self._node = LazyNode.leaf(array.copy() if copy else array,
                                   cache_native=copy)
        self.requires_grad = bool(requires_grad)
        self.grad: Optional[Tensor] = None
        self._is_leaf = True

    @classmethod
    def _wrap(cls, node: LazyNode, requires_grad: bool = False) -> "Tensor":
        made = cls.__new__(cls)
        made._node = node
        made.requires_grad = requires_grad
        made.grad = None
        made._is_leaf = False
        return made

    @classmethod
    def from_native(cls, value: object, *, backend: str, shape: Sequence[int],
                    dtype: np.dtype) -> "Tensor":
        """Wrap backend-owned storage without copying (tensor.py:82-102)."""
        if not backend:
            raise ValueError("backend name cannot be empty")
        dims = tuple(int(n) for n in shape)
        if any(n < 0 for n in dims):
            raise ValueError("native tensor dimensions cannot be negative")
        made = cls._wrap(LazyNode.native_leaf(backend, value, dims, np.dtype(dtype)))
        made._is_leaf = True
        return made

    @classmethod
    def zeros(cls, shape: Sequence[int], *, dtype: np.dtype = np.float32) -> "Tensor":
        return cls(np.zeros(tuple(shape), dtype=dtype), copy=False)

    @classmethod
    def ones(cls, shape: Sequence[int], *, dtype: np.dtype = np.float32) -> "Tensor":
        return cls(np.ones(tuple(shape), dtype=dtype), copy=False)

    # -- metadata -----------------------------------------------------------
    @property
    def shape(self) -> Tuple[int, ...]:
        return self._node.shape

    @property
    def ndim(self) -> int:
        return len(self._node.shape)

    @property
    def dtype(self) -> np.dtype:
        return self._node.dtype

    @property
    def T(self) -> "Tensor":
        if self.ndim != 2:
            raise ValueError("T is only defined for 2D tensors; use permute instead")
        return self.permute(1, 0)

    def numpy(self, compiler: Optional[str] = None) -> np.ndarray:
        return realize(self, compiler=compiler)[0]

    def item(self, compiler: Optional[str] = None) -> object:
        if self.shape != ():
            raise ValueError("item() requires a scalar tensor")
        return self.numpy(compiler).item()

    def detach(self) -> "Tensor":
        return Tensor._wrap(self._node)

    def backward(self, grad: Optional[ArrayLike] = None) -> None:
        raise NotImplementedError(
            "cuda-b200 accelerates inference; training graphs are not supported"
        )

    # -- elementwise --------------------------------------------------------
    def _lift(self, other: Union["Tensor", ArrayLike]) -> "Tensor":
        """Python/NumPy operands become leaves of *this* tensor's dtype (tensor.py:205-208)."""
        return other if isinstance(other, Tensor) else Tensor(other, dtype=self.dtype)

    def _binary(self, other: Union["Tensor", ArrayLike], kind: str) -> "Tensor":
        rhs = self._lift(other)
        node = LazyNode(Op.ELEMENTWISE, (self._node, rhs._node), kind,
                        np.broadcast_shapes(self.shape, rhs.shape),
                        np.result_type(self.dtype, rhs.dtype))
        return Tensor._wrap(node)

    def _unary(self, kind: str) -> "Tensor":
        return Tensor._wrap(LazyNode(Op.ELEMENTWISE, (self._node,), kind,
                                     self.shape, self.dtype))

    def __add__(self, other): return self._binary(other, "add")
    def __radd__(self, other): return self + other
    def __sub__(self, other): return self._binary(other, "sub")
    def __rsub__(self, other): return self._lift(other) - self
    def __mul__(self, other): return self._binary(other, "mul")
    def __rmul__(self, other): return self * other
    def __truediv__(self, other): return self._binary(other, "div")
    def __rtruediv__(self, other): return self._lift(other) / self
    def __neg__(self): return self._unary("neg")

    def equal(self, other: Union["Tensor", ArrayLike]) -> "Tensor":
        return self._binary(other, "equal")

    def exp(self) -> "Tensor": return self._unary("exp")
    def log(self) -> "Tensor": return self._unary("log")
    def relu(self) -> "Tensor": return self._unary("relu")
    def sqrt(self) -> "Tensor": return self._unary("sqrt")

    def softmax(self, axis: int = -1) -> "Tensor":
        """max-shift, exp, sum, divide; lowering hint ``softmax`` (tensor.py:325-334)."""
        which = _axes(axis, self.ndim)[0]
        peak = self.max(axis=axis, keepdims=True).detach()
        raised = (self - peak).exp()
        result = raised / raised.sum(axis=axis, keepdims=True)
        result._node.lowering = ("softmax", (self._node,), which)
        return result

    def log_softmax(self, axis: int = -1) -> "Tensor":
        """Lowering hint ``log_softmax`` (tensor.py:426-435)."""
        which = _axes(axis, self.ndim)[0]
        peak = self.max(axis=axis, keepdims=True).detach()
        shifted = self - peak
        result = shifted - shifted.exp().sum(axis=axis, keepdims=True).log()
        result._node.lowering = ("log_softmax", (self._node,), which)
        return result

    # -- movement -----------------------------------------------------------
    def reshape(self, *shape: Union[int, Sequence[int]]) -> "Tensor":
        wanted = list(shape[0]) if len(shape) == 1 and not isinstance(shape[0], int) else list(shape)
        if wanted.count(-1) > 1:
            raise ValueError("only one inferred dimension is allowed")
        total = int(np.prod(self.shape))
        if -1 in wanted:
            known = int(np.prod([n for n in wanted if n != -1]))
            if known == 0 or total % known:
                raise ValueError("shape is not compatible with tensor size")
            wanted[wanted.index(-1)] = total // known
        final = tuple(int(n) for n in wanted)
        if int(np.prod(final)) != total:
            raise ValueError("shape is not compatible with tensor size")
        return Tensor._wrap(LazyNode(Op.RESHAPE, (self._node,), final, final, self.dtype))

    def permute(self, *axes: int) -> "Tensor":
        if len(axes) != self.ndim or set(axes) != set(range(self.ndim)):
            raise ValueError(f"expected a permutation of {tuple(range(self.ndim))}")
        shape = tuple(self.shape[a] for a in axes)
        return Tensor._wrap(LazyNode(Op.PERMUTE, (self._node,), tuple(axes), shape,
                                     self.dtype))

    def transpose(self, dim0: int, dim1: int) -> "Tensor":
        a = dim0 + self.ndim if dim0 < 0 else dim0
        b = dim1 + self.ndim if dim1 < 0 else dim1
        if not (0 <= a < self.ndim and 0 <= b < self.ndim):
            raise ValueError(f"invalid transpose dimensions {dim0}, {dim1}")
        order = list(range(self.ndim))
        order[a], order[b] = order[b], order[a]
        return self.permute(*order)

    # -- contraction / indexing / reduction --------------------------------
    def __matmul__(self, other: "Tensor") -> "Tensor":
        if not isinstance(other, Tensor):
            raise TypeError("matmul requires another Tensor")
        if self.ndim < 2 or other.ndim < 2:
            raise ValueError("matmul requires tensors with at least two dimensions")
        if self.shape[-1] != other.shape[-2]:
            raise ValueError(f"cannot multiply shapes {self.shape} and {other.shape}")
        batch = np.broadcast_shapes(self.shape[:-2], other.shape[:-2])
        shape = batch + (self.shape[-2], other.shape[-1])
        return Tensor._wrap(LazyNode(Op.MATMUL, (self._node, other._node), None, shape,
                                     np.result_type(self.dtype, other.dtype)))

    def gather(self, indices: "Tensor") -> "Tensor":
        """Rows of ``self`` selected by integer ``indices`` (tensor.py:527-544)."""
        if not isinstance(indices, Tensor):
            raise TypeError("gather indices must be a Tensor")
        if not np.issubdtype(indices.dtype, np.integer):
            raise TypeError("gather indices must have an integer dtype")
        shape = indices.shape + self.shape[1:]
        return Tensor._wrap(LazyNode(Op.GATHER, (self._node, indices._node), None,
                                     shape, self.dtype))

    def _reduce(self, kind: str, axis: Axis, keepdims: bool) -> "Tensor":
        axes = _axes(axis, self.ndim)
        return Tensor._wrap(LazyNode(Op.REDUCE, (self._node,), (kind, axes, keepdims),
                                     _kept(self.shape, axes, keepdims), self.dtype))

    def sum(self, axis: Axis = None, keepdims: bool = False) -> "Tensor":
        return self._reduce("sum", axis, keepdims)

    def mean(self, axis: Axis = None, keepdims: bool = False) -> "Tensor":
        axes = _axes(axis, self.ndim)
        count = int(np.prod([self.shape[a] for a in axes]))
        return self.sum(axis=axes, keepdims=keepdims) / count

    def max(self, axis: Axis = None, keepdims: bool = False) -> "Tensor":
        return self._reduce("max", axis, keepdims)

    def __repr__(self) -> str:
        kind = "leaf" if self._is_leaf else "lazy"
        return (f"Tensor(shape={self.shape}, dtype={self.dtype}, "
                f"requires_grad={self.requires_grad}, {kind})")


def realize(*tensors: Tensor, compiler: Optional[str] = None) -> Tuple[np.ndarray, ...]:
    return compile_graph(*tensors, compiler=compiler)()


def compile_graph(*tensors: Tensor, compiler: Optional[str] = None,
                  dynamic_inputs: Sequence[Tensor] = ()) -> CompiledProgram:
    """Compile output tensors with a registered plugin (tensor.py:629-642)."""
    if not tensors:
        raise ValueError("at least one tensor is required")
    chosen = get_compiler(compiler)
    outputs = [t._node for t in tensors]
    if not dynamic_inputs:
        return chosen.compile(outputs)
    return chosen.compile(outputs, [t._node for t in dynamic_inputs])
