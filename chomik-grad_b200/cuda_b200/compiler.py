"""``CudaB200Compiler``: the ``cuda-b200`` plugin's ``Compiler``.

Implements ``Compiler.compile(outputs, dynamic_inputs=())``
(chomikgrad/lazy.py:172-183) with the reference CUDA plugin's conventions
(``cache_size``, ``close()``, errors: cuda_backend.py:385-453):

* ``ValueError`` for an empty output list, a non-leaf dynamic input, or a
  dynamic input that is not a leaf of the compiled graph (dynamic inputs that
  a lowering prunes, e.g. the decode RoPE ``rotation``, are accepted and
  ignored, like mlx_backend.py:249-258);
* ``TypeError`` for dtypes the kernels do not implement (float64, ...);
* ``RuntimeError`` when no B200 is present -- never a CPU fallback.
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

from . import _lib
from .device import CudaB200Device, DeviceArray
from chomikgrad.lazy import Compiler
from .planner import Planner
from .program import CudaB200Program


class CudaB200Compiler(Compiler):
    """Lower chomik-grad graphs to sm_100a kernels (see cuda_b200.planner)."""

    name = "cuda-b200"

    def __init__(self, device_index: Optional[int] = None, *, use_graphs: Optional[bool] = None,
                 pdl: bool = True, fuse_decode: bool = True, alias_caches: bool = True,
                 max_positions: int = 8192, gemv_grid: Optional[int] = None,
                 decode_step: Optional[bool] = None, gemm_min_rows: Optional[int] = None,
                 attn_min_rows: Optional[int] = None, kv_cache_dtype: Optional[str] = None) -> None:
        import os

        self.device = CudaB200Device(device_index)
        if gemv_grid is None:  # CTAs per decode GEMV (0 = one per SM)
            gemv_grid = int(os.environ.get("CUDA_B200_GEMV_GRID", "0"))
        if use_graphs is None:  # CUDA graphs for repeated runs (CUDA_B200_GRAPHS=0: launch one by one)
            use_graphs = os.environ.get("CUDA_B200_GRAPHS", "1") != "0"
        if decode_step is None:  # fused decode steps as one persistent launch (cb_decode_step)
            decode_step = os.environ.get("CUDA_B200_DECODE_STEP", "1") != "0"
        self.decode_step = decode_step
        if gemm_min_rows is None:  # rows from which x @ W.T runs on the tcgen05 GEMM (cb_gemm_tc)
            gemm_min_rows = int(os.environ.get("CUDA_B200_GEMM_MIN_ROWS", "64"))
        self.gemm_min_rows = gemm_min_rows
        if attn_min_rows is None:  # query rows from which attention runs on cb_sdpa_tc
            attn_min_rows = int(os.environ.get("CUDA_B200_ATTN_MIN_ROWS", "64"))
        self.attn_min_rows = attn_min_rows
        # KV caches produced by prefill and updated by decode: float32 (the
        # runtime dtype of the reference's caches, the default) or bfloat16
        # (CUDA_B200_KV_DTYPE=bfloat16): half the attention's bytes; the rows
        # a step writes are rounded to bfloat16.
        if kv_cache_dtype is None:
            kv_cache_dtype = os.environ.get("CUDA_B200_KV_DTYPE", "float32")
        if kv_cache_dtype not in ("float32", "bfloat16"):
            raise ValueError(f"kv_cache_dtype must be float32 or bfloat16, not {kv_cache_dtype!r}")
        self.kv_cache_dtype = kv_cache_dtype
        # cb_decode_step_prepare flags: attention splits are merged in the
        # attention phase (measured faster on TinyLlama); set
        # CUDA_B200_STEP_MERGE=stage to merge them in the O projection's x staging
        self.step_flags = _lib.STEP_MERGE_IN_STAGE if os.environ.get("CUDA_B200_STEP_MERGE") == "stage" else 0
        self.use_graphs = use_graphs
        self.pdl = pdl
        self.fuse_decode = fuse_decode
        self.alias_caches = alias_caches
        self.max_positions = max_positions
        self.gemv_grid = gemv_grid
        self._tables: dict = {}
        self._programs: list = []

    @property
    def cache_size(self) -> int:
        return 0

    def close(self) -> None:
        self.device.synchronize()
        for program in self._programs:
            program.close()
        self._programs.clear()
        self._tables.clear()

    def _leaf_dtype(self, node) -> np.dtype:
        native = node.native_values.get(self.device.name)
        if isinstance(native, DeviceArray):
            return native.dtype
        if node.value is not None:
            return np.asarray(node.value).dtype
        return np.asarray(node.numpy_value()).dtype

    def plan(self, outputs: Sequence[object], dynamic_inputs: Sequence[object] = ()):
        """Planning only (host side); exposed for inspection and tests."""
        if not outputs:
            raise ValueError("at least one output is required")
        if any(node.op is not None for node in dynamic_inputs):
            raise ValueError("dynamic inputs must be graph leaves")
        return Planner(outputs, dynamic_inputs, backend=self.device.name,
                       leaf_dtype=self._leaf_dtype, max_positions=self.max_positions,
                       fuse_decode=self.fuse_decode, alias_caches=self.alias_caches,
                       table_cache=self._tables, gemm_min_rows=self.gemm_min_rows,
                       kv_bf16=self.kv_cache_dtype == "bfloat16").build()

    def compile(self, outputs: Sequence[object],
                dynamic_inputs: Sequence[object] = ()) -> CudaB200Program:
        program = CudaB200Program(self.plan(outputs, dynamic_inputs), self)
        return program

    # ------------------------------------------------------------ training
    def update_parameters(self, parameters: Sequence[object], gradients: Sequence[object], learning_rate: float,
                          *, inplace: bool = False):
        """SGD step (``SGD.step``, chomikgrad/optim.py:28-64): the gradients' graph compiled and run
        on the device, then :meth:`update_native_parameters`."""
        if len(parameters) != len(gradients):
            raise ValueError("parameter and gradient counts must match")
        native = self.compile(list(gradients)).run(synchronize=False) if gradients else []
        return self.update_native_parameters(parameters, native, learning_rate, inplace=inplace)

    def update_native_parameters(self, parameters: Sequence[object], gradients: Sequence[object],
                                 learning_rate: float, *, inplace: bool = False):
        """``param - lr * grad`` for float32 parameters, up to ``_lib.SGD_GROUP`` tensors per launch
        (``cb_sgd_update``).  Returns new leaves holding the updated parameters (in place: the
        parameters' own storage) and the gradients (Compiler.update_native_parameters,
        chomikgrad/lazy.py:199-209; compiled training steps, chomikgrad/jit.py:113-160)."""
        import ctypes

        import torch
        from chomikgrad.lazy import LazyNode

        if len(parameters) != len(gradients):
            raise ValueError("parameter and gradient counts must match")
        natives, grads = [], []
        for node, grad in zip(parameters, gradients):
            native = node.native_values.get(self.device.name)
            if not isinstance(native, DeviceArray):
                native = self.device.array(node.numpy_value())
                if node.cache_native:
                    node.native_values[self.device.name] = native
            grad = self.device.array(grad)
            if native.dtype != np.float32 or grad.dtype != np.float32:
                raise TypeError("cuda-b200 updates float32 parameters with float32 gradients")
            if native.size != grad.size or tuple(native.shape) != tuple(node.shape):
                raise ValueError("gradient shape does not match parameter shape")
            natives.append(native)
            grads.append(grad)
        outs = natives if inplace else [DeviceArray(torch.empty_like(p.tensor), p.shape, p.dtype) for p in natives]
        stream = self.device.stream()
        for start in range(0, len(natives), _lib.SGD_GROUP):
            group = _lib.SgdGroup()
            chunk = range(start, min(start + _lib.SGD_GROUP, len(natives)))
            group.n = len(chunk)
            group.lr = float(np.float32(learning_rate))
            for j, i in enumerate(chunk):
                group.param[j] = natives[i].data_ptr()
                group.grad[j] = grads[i].data_ptr()
                group.out[j] = outs[i].data_ptr()
                group.count[j] = natives[i].size
            _lib.call("cb_sgd_update", ctypes.byref(group), stream)
        name = self.device.name
        parameter_nodes = tuple(LazyNode.native_leaf(name, out, node.shape, node.dtype)
                                for node, out in zip(parameters, outs))
        gradient_nodes = tuple(LazyNode.native_leaf(name, grad, node.shape, node.dtype)
                               for node, grad in zip(parameters, grads))
        return parameter_nodes, gradient_nodes
