"""Execution of a :class:`~cuda_b200.planner.Plan` on the GPU.

A program owns a static set of device buffers (intermediates, tables,
scratch, and slots for inputs that are copied in), so its launch sequence has
fixed pointers and is recorded once into a CUDA graph and replayed: one
``cudaGraphLaunch`` per ``run`` instead of the reference's per-node Python
dispatch (chomikgrad/lazy.py:487-492, cuda_backend.py:55-69).

Input binding follows ``CompiledProgram.run`` (chomikgrad/lazy.py:158-165):
bound dynamic inputs are used for this run only, unbound leaves use their
cached native value or upload their host value (cache_native leaves once,
others every run, so host mutation of ``copy=False`` tensors is observed).
Small inputs are copied into program-owned slots; KV caches that the plan
updates in place are bound by pointer and returned as the same objects.
Other outputs are fresh arrays owned by the caller.

Graphs are keyed by the addresses of pointer-bound inputs; a key seen twice
is captured and replayed from then on.

A fused decode step (only GEMV and decode-attention steps) runs as ONE
persistent launch, ``cb_decode_step``, instead of one launch per step: the
steps become the phases of its table (prepared per key, since the table holds
the bound pointers).  The SwiGLU epilogue of a gate/up GEMV becomes a plain
store of [gate | up] into a program buffer plus the SwiGLU x mode of the
down-projection phase that reads it.
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from .device import DeviceArray, torch_dtype
from chomikgrad.lazy import CompiledProgram
from .planner import Buffer, Plan, Step, View, bf16, contiguous_strides, gemm_shape  # noqa: F401

_BF16 = bf16()
_UNBOUND = object()  # a leaf without a binding in this run


def _torch():
    import torch

    return torch


class CudaB200Program(CompiledProgram):
    """A compiled graph: static buffers + a replayable launch sequence."""

    def __init__(self, plan: Plan, compiler) -> None:
        self.plan = plan
        self.source = plan.source
        self.inputs = plan.inputs
        self.device = compiler.device
        self._compiler = compiler
        self._built = False
        self._tensors: Dict[Buffer, object] = {}
        self._ptr: Dict[Buffer, int] = {}
        self._graphs: Dict[tuple, int] = {}
        self._seen: Dict[tuple, int] = {}
        self._capture_stream: Optional[int] = None
        self.use_graphs = compiler.use_graphs
        self.launches = 0  # kernels launched by the last eager run (graph replays re-run them)
        self.step_mode = bool(getattr(compiler, "decode_step", False)) and self._fusable(plan, self.device.sm_count)
        # constants the plan was specialised on, once per leaf (a shared leaf,
        # e.g. the GQA broadcast's ones, is guarded by every layer that uses it)
        guards: Dict[int, tuple] = {}
        for leaf, expected in plan.guards:
            guards.setdefault(id(leaf), (leaf, np.ascontiguousarray(expected)))
        self._guards = list(guards.values())
        self._step_tables: Dict[tuple, Tuple[object, _lib.DecodeStepConfig]] = {}

    @staticmethod
    def _fusable(plan: Plan, sms: int) -> bool:
        """Whether the plan is a fused decode step cb_decode_step can run whole.

        Its consumer threads stage at most 3 x 256 vectors of x per phase
        (6144 bf16-weight or 3072 float32-weight columns), and a block (one
        per SM) owns at most 128 SwiGLU gate/up pairs; a plan with a wider
        GEMV (the Llama-3-8B down projection, 14336 columns) runs kernel by
        kernel.
        """
        names = {s.name for s in plan.steps}
        if not (plan.steps and names <= {"gemv", "decode_attention"} and "gemv" in names):
            return False
        for s in plan.steps:
            if s.name != "gemv":
                continue
            elems = 8 if s.args["weights"][0].dtype.itemsize == 2 else 4
            if s.args["k"] > _lib.STEP_X_VECTORS * elems:
                return False
            if s.args["epilogue"] == _lib.EPI_SILU_MUL and -(-s.args["rows"][0] // sms) > _lib.STEP_ROWS_PER_BLOCK:
                return False
        return True

    # ------------------------------------------------------------ build
    def _build(self) -> None:
        torch = _torch()
        dev = self.device.torch_device
        # Copy-bound inputs (the small per-step ones) live in one device arena
        # mirrored by a pinned host block: a step's host inputs are written
        # into the mirror and reach their slots in one asynchronous copy.
        arena_off: Dict[Buffer, int] = {}
        top = 0
        for buf in self.plan.buffers:
            if buf.kind == "input" and buf.bind == "copy":
                arena_off[buf] = top
                top += (max(buf.size, 1) * buf.dtype.itemsize + 15) // 16 * 16
        self._arena = torch.empty(max(top, 16), dtype=torch.uint8, device=dev)
        self._staging = torch.empty(max(top, 16), dtype=torch.uint8, pin_memory=True)
        self._staging_np = self._staging.numpy()
        self._staging_done = None  # event after the last staged copy (the mirror is reused)
        self._arena_off = arena_off
        for buf, off in arena_off.items():
            count = max(buf.size, 1)
            view = self._arena[off: off + count * buf.dtype.itemsize]
            tensor = view.view(torch_dtype(buf.dtype)) if buf.dtype.name != "bfloat16" else \
                view.view(torch.int16).view(torch.bfloat16)
            self._tensors[buf] = tensor
            self._ptr[buf] = int(tensor.data_ptr())
        for buf in self.plan.buffers:
            if buf.kind == "input" and buf.bind == "pointer":
                continue  # bound per run
            if buf in arena_off:
                continue
            if buf.kind == "aux" and buf.host is not None:
                arr = self.device.array(buf.host)
                self._tensors[buf] = arr.tensor
            else:
                count = max(buf.size, 1)
                tensor = (torch.zeros if buf.zero else torch.empty)(
                    count, dtype=torch_dtype(buf.dtype), device=dev)
                self._tensors[buf] = tensor
            self._ptr[buf] = int(self._tensors[buf].data_ptr())
        self._bind_constants()
        stream = self.device.stream()
        for init in self.plan.init_steps:
            if init["name"] == "rms_table":
                self._rms_table(init, stream)
        if self.step_mode:
            n = len(self.plan.steps)
            self._step_counters = torch.zeros(n, dtype=torch.int32, device=dev)
            self._step_flag = (self._tensors[self.plan.error_flag] if self.plan.error_flag is not None
                               else torch.zeros(1, dtype=torch.int32, device=dev))
        self._group_row_matmuls()
        rows_scratch, n_counters = [0], 0
        for leader, group in self._rows.items():
            args = self._rows_args(group, counters=0)
            rows_scratch.append(int(_lib.load().cb_gemm_rows_scratch(ctypes.byref(args))))
            self._rows_counter_off[leader] = n_counters
            n_counters += int(_lib.load().cb_gemm_rows_counters(ctypes.byref(args)))
        for step in self.plan.steps:  # fused row GEMMs (planner's matmul_rows)
            if step.name != "matmul_rows":
                continue
            args = self._matmul_rows_args(step, counters=0)
            rows_scratch.append(int(_lib.load().cb_gemm_rows_scratch(ctypes.byref(args))))
            self._rows_counter_off[id(step)] = n_counters
            n_counters += int(_lib.load().cb_gemm_rows_counters(ctypes.byref(args)))
        self._rows_counters = torch.zeros(max(n_counters, 1), dtype=torch.int32, device=dev)
        scratch = max([self._gemm_scratch_bytes(s) for s in self.plan.steps if s.name == "matmul"] +
                      [self._multi_scratch_bytes(s) for s in self.plan.steps if s.name == "matmul_multi"] +
                      [self._sdpa_scratch_bytes(s) for s in self.plan.steps if s.name == "sdpa"] + rows_scratch)
        self._gemm_scratch = torch.empty(max(scratch, 16), dtype=torch.uint8, device=dev)
        self._gemm_flag = (self._tensors[self.plan.error_flag] if self.plan.error_flag is not None
                           else torch.zeros(1, dtype=torch.int32, device=dev))
        self._built = True

    def _rms_table(self, init, stream: int) -> None:
        table: View = init["table"]
        spec = init["spec"]
        leaf_ptr = self._leaf_pointer(table.buf)
        args = self._rms_args(leaf_ptr, table.dtype, table.shape[0], table.shape[1], spec)
        _lib.call("cb_rmsnorm_row_table", ctypes.byref(args), self._ptr[init["out"]], stream)

    # ------------------------------------------------------------ inputs
    def _load(self, leaf) -> DeviceArray:
        """Native value of an unbound leaf (lazy.py:94-104; cuda_backend.py:395-401)."""
        name = self.device.name
        native = leaf.native_values.get(name)
        if native is not None:
            return native
        arr = self.device.array(leaf.numpy_value())
        if leaf.cache_native:
            leaf.native_values[name] = arr
        return arr

    def _leaf_pointer(self, buf: Buffer) -> int:
        if buf in self._ptr:
            return self._ptr[buf]
        return self._load(buf.node).data_ptr()

    def _bind_constants(self) -> None:
        """Resolve immutable (cache_native, non-dynamic) leaves once per program."""
        self._constants = {}
        self._per_run = []
        for leaf, buf in self.plan.input_buffers.items():
            if buf.bind == "pointer" and leaf.cache_native and leaf not in self.plan.dynamic:
                arr = self._load(leaf)
                self._check(arr, buf)
                self._constants[leaf] = arr
                self._ptr[buf] = arr.data_ptr()
            else:
                self._per_run.append((leaf, buf))
        self._last_bound: List[Optional[Tuple[DeviceArray, int]]] = [None] * len(self._per_run)

    @staticmethod
    def _check(arr: DeviceArray, buf: Buffer) -> None:
        if arr.shape != tuple(buf.shape):
            raise ValueError(f"input bound with shape {arr.shape}, program expects {buf.shape}")
        if arr.dtype != buf.dtype:
            raise TypeError(f"input bound with dtype {arr.dtype}, program was compiled for "
                            f"{buf.dtype}; compile a new program for this dtype")

    def _bind(self, bindings: Mapping) -> Tuple[Dict[object, DeviceArray], tuple]:
        """Per-run inputs: pointers of pointer-bound leaves, host values into the input slots.

        A pointer-bound leaf rebound with the very DeviceArray it had last
        run (the caches a decode step returned, bound to the next step) keeps
        its checked pointer without re-checking.
        """
        bound: Dict[object, DeviceArray] = {}
        key = []
        device_copies = []
        staged = False
        last = self._last_bound
        for i, (leaf, buf) in enumerate(self._per_run):
            value = bindings.get(leaf, _UNBOUND)
            if buf.bind == "pointer":
                prev = last[i]
                if prev is not None and value is prev[0]:
                    arr, ptr = prev
                else:
                    arr = self.device.array(value) if value is not _UNBOUND else self._load(leaf)
                    self._check(arr, buf)
                    ptr = arr.data_ptr()
                    last[i] = (arr, ptr) if value is arr else None
                bound[leaf] = arr
                self._ptr[buf] = ptr
                key.append(ptr)
                continue
            arr = self.device.array(value) if value is not _UNBOUND else self._load(leaf)
            self._check(arr, buf)
            bound[leaf] = arr
            if arr.size == 0:
                continue
            elif arr.host is not None:  # pending host input: through the pinned mirror
                if not staged and self._staging_done is not None:
                    self._staging_done.synchronize()  # the previous step's copy has read the mirror
                staged = True
                host = np.ascontiguousarray(arr.host).reshape(-1)
                off = self._arena_off[buf]
                self._staging_np[off: off + host.nbytes] = host.view(np.uint8)
            else:
                device_copies.append((buf, arr))
        if staged:
            torch = _torch()
            self._arena.copy_(self._staging, non_blocking=True)
            if self._staging_done is None:
                self._staging_done = torch.cuda.Event()
            self._staging_done.record()
        for buf, arr in device_copies:  # after the mirror copy, which covers every slot
            n = max(buf.size, 1)
            self._tensors[buf][:n].copy_(arr.tensor[:n], non_blocking=True)
        return bound, tuple(key)

    # ------------------------------------------------------------ run
    def run(self, bindings: Optional[Mapping] = None, *, synchronize: bool = False) -> Tuple[object, ...]:
        torch = _torch()
        with torch.cuda.device(self.device.torch_device):
            if not self._built:
                self._build()
            for leaf, expected in self._guards:
                value = np.asarray(leaf.numpy_value())
                if (value.shape != expected.shape or value.dtype != expected.dtype
                        or value.tobytes() != expected.tobytes()):
                    raise RuntimeError("a constant the program was specialised on has changed; "
                                       "compile the graph again")
            bound, key = self._bind(bindings or {})
            self._last_key = key
            stream = self.device.stream()
            exec_ = self._graphs.get(key)
            if exec_ is not None:
                _lib.call("cb_graph_launch", exec_, stream)
            else:
                self._seen[key] = self._seen.get(key, 0) + 1
                if self.use_graphs and self._seen[key] >= 2 and len(self._graphs) < 8:
                    if self.step_mode:
                        self._step_table()  # prepared outside the capture (it copies and synchronises)
                    exec_ = self._capture()
                    self._graphs[key] = exec_
                    _lib.call("cb_graph_launch", exec_, stream)
                else:
                    self._launch_all(stream)
            outputs = self._collect(bound)
            if synchronize:
                self.device.synchronize()
                self.check_errors()
        return outputs

    # ------------------------------------------------ device-side driving
    def slot_pointer(self, leaf) -> int:
        """Device address of the program-owned slot a small dynamic input is copied into."""
        buf = self.plan.input_buffers[leaf]
        if buf.bind != "copy":
            raise ValueError("this input is bound by pointer, it has no slot")
        return self._ptr[buf]

    def argmax_pointer(self, output_index: int = 0) -> int:
        """Device address of the int64 argmax the program computes for an output."""
        return self._ptr[self.plan.argmax_of[output_index]]

    def error_pointer(self) -> int:
        return self._ptr[self.plan.error_flag] if self.plan.error_flag is not None else 0

    def replay(self, stream: Optional[int] = None) -> None:
        """Re-run the captured graph of the last ``run`` on the current slot contents.

        No inputs are bound and no outputs are copied out: device-side drivers
        (cb_decode_advance) update the slots between replays.
        """
        stream = self.device.stream() if stream is None else stream
        if not self.use_graphs:  # graphs switched off: launch the same kernels one by one
            self._launch_all(stream)
            return
        exec_ = self._graphs.get(getattr(self, "_last_key", None))
        if exec_ is None:
            raise RuntimeError("replay() needs a captured graph: run() the program twice first")
        _lib.call("cb_graph_launch", exec_, stream)

    def _capture(self) -> int:
        if self._capture_stream is None:
            s = ctypes.c_void_p()
            _lib.call("cb_stream_create", ctypes.byref(s))
            self._capture_stream = s.value
        # the capture stream must see all prior work of the current stream
        self.device.synchronize()
        _lib.call("cb_capture_begin", self._capture_stream)
        try:
            self._launch_all(self._capture_stream)
        finally:
            exec_ = ctypes.c_void_p()
            status = _lib.load().cb_capture_end(self._capture_stream, ctypes.byref(exec_))
        _lib.check(status, "cb_capture_end")
        return exec_.value

    def _collect(self, bound: Dict[object, DeviceArray]) -> Tuple[object, ...]:
        torch = _torch()
        outs: List[DeviceArray] = []
        for index, (node, view) in enumerate(self.plan.outputs):
            alias = self.plan.aliases.get(index)
            if alias is not None:
                outs.append(bound[alias])
                continue
            if node.op is None and (node in bound or node in self._constants):
                outs.append(bound[node] if node in bound else self._constants[node])
                continue
            outs.append(self._copy_out(view, node.shape))
            argmax = self.plan.argmax_of.get(index)
            if argmax is not None:
                status = torch.empty(2, dtype=torch.int64, device=self.device.torch_device)
                status[:1].copy_(self._tensors[argmax][:1])
                if self.plan.error_flag is not None:
                    status[1:].copy_(self._tensors[self.plan.error_flag][:1])
                else:
                    status[1:].zero_()
                outs[-1].argmax_value = status
        return tuple(outs)

    def _copy_out(self, view: View, shape) -> DeviceArray:
        torch = _torch()
        count = int(np.prod(shape)) if len(shape) else 1
        out = torch.empty(max(count, 1), dtype=torch_dtype(view.dtype), device=self.device.torch_device)
        base = self._ptr.get(view.buf)
        if base is None:
            base = self._leaf_pointer(view.buf)
        if count:
            if view.is_contiguous():
                src = self._tensors.get(view.buf)
                if src is not None:
                    out[:count].copy_(src[view.offset: view.offset + count])
                else:
                    _lib.call("cb_copy_strided", base, view.offset, out.data_ptr(),
                              view.dtype.itemsize, 1, _lib.ll_array([count]), _lib.ll_array([1]),
                              self.device.stream())
            else:
                _lib.call("cb_copy_strided", base, view.offset, out.data_ptr(), view.dtype.itemsize,
                          len(view.shape), _lib.ll_array(view.shape), _lib.ll_array(view.strides),
                          self.device.stream())
        return DeviceArray(out, tuple(shape), view.dtype)

    def check_errors(self) -> None:
        """Raise if a kernel set the program's error flag (cb_gemv_args.error_flag)."""
        if self.step_mode and self._built:
            flag = self._step_flag
        elif self.plan.error_flag is not None:
            flag = self._tensors[self.plan.error_flag]
        elif self._built:
            flag = self._gemm_flag
        else:
            return
        value = int(flag[0].item())
        if value:
            flag.zero_()
            if value >= _lib.FLAG_WAIT_DATA:
                self._reset_counters()
            raise _lib.flag_error(value)

    # ------------------------------------------------------------ launches
    def ptr(self, view: View) -> int:
        base = self._ptr.get(view.buf)
        if base is None:
            base = self._leaf_pointer(view.buf)
        return base + view.offset * view.dtype.itemsize

    def _launch_all(self, stream: int) -> None:
        if self.step_mode:
            self._launch_step(stream)
            return
        self._extra_launches = 0  # kernels beyond one per step (the GEMM's plane split)
        for step in self.plan.steps:
            getattr(self, f"_step_{step.name}")(step, stream)
        self.launches = len(self.plan.steps) + self._extra_launches

    def _step_copy(self, step: Step, stream: int) -> None:
        src: View = step.args["src"]
        if src.size == 0:
            return
        _lib.call("cb_copy_strided", self.ptr(src), 0, self.ptr(step.out), src.dtype.itemsize,
                  len(src.shape), _lib.ll_array(src.shape), _lib.ll_array(src.strides), stream)

    def _step_elementwise(self, step: Step, stream: int) -> None:
        shape = step.args["shape"]
        nd = len(shape)
        a = _lib.ElementwiseArgs()
        a.ndim = nd
        a.out_dtype = _lib.dtype_code(step.out.dtype)
        for d, n in enumerate(shape):
            a.shape[d] = n
        views: Sequence[View] = step.args["inputs"]
        a.n_inputs = len(views)
        for i, v in enumerate(views):
            a.inputs[i] = self.ptr(v)
            a.in_dtype[i] = _lib.dtype_code(v.dtype)
            a.in_offset[i] = 0
            lead = nd - len(v.shape)
            for d in range(nd):
                j = d - lead
                a.in_strides[i][d] = 0 if j < 0 or v.shape[j] == 1 else v.strides[j]
        instrs = step.args["instrs"]
        a.n_instr = len(instrs)
        for t, (name, lhs, rhs, dt) in enumerate(instrs):
            a.op[t] = _lib.OPS[name]
            a.lhs[t] = lhs
            a.rhs[t] = rhs
            a.round[t] = _lib.dtype_code(dt)
        a.out = self.ptr(step.out)
        _lib.call("cb_elementwise", ctypes.byref(a), stream)

    # ------------------------------------------------------------ training lowerings
    def _step_softmax(self, step: Step, stream: int) -> None:
        a = step.args
        _lib.call("cb_softmax_rows", self.ptr(a["x"]), a["rows"], a["width"], int(a["log"]), self.ptr(step.out),
                  stream)

    def _step_softmax_backward(self, step: Step, stream: int) -> None:
        a = step.args
        _lib.call("cb_softmax_backward_rows", self.ptr(a["grad"]), self.ptr(a["y"]), a["rows"], a["width"],
                  int(a["log"]), self.ptr(step.out), stream)

    def _step_layer_norm(self, step: Step, stream: int) -> None:
        a = step.args
        _lib.call("cb_layer_norm_rows", self.ptr(a["x"]), self.ptr(a["w"]), self.ptr(a["b"]), a["rows"], a["width"],
                  a["eps"], self.ptr(step.out), stream)

    def _step_layer_norm_backward(self, step: Step, stream: int) -> None:
        a = step.args
        opt = lambda v: None if v is None else self.ptr(v)  # noqa: E731
        stats = None if a["stats"] is None else self._ptr[a["stats"]]
        _lib.call("cb_layer_norm_backward_rows", self.ptr(a["grad"]), self.ptr(a["x"]), self.ptr(a["w"]), a["rows"],
                  a["width"], a["eps"], opt(a["dx"]), opt(a["dw"]), opt(a["db"]), stats, stream)

    def _add_into(self, out: View, residual: View, stream: int) -> None:
        """out = residual + out (both contiguous, the same shape), in place."""
        a = _lib.ElementwiseArgs()
        a.ndim, a.out_dtype, a.n_inputs, a.n_instr = 1, _lib.dtype_code(out.dtype), 2, 1
        a.shape[0] = out.size
        for i, v in enumerate((residual, out)):
            a.inputs[i] = self.ptr(v)
            a.in_dtype[i] = _lib.dtype_code(v.dtype)
            a.in_offset[i] = 0
            a.in_strides[i][0] = 1
        a.op[0], a.lhs[0], a.rhs[0], a.round[0] = _lib.OPS["add"], 0, 1, _lib.F32
        a.out = self.ptr(out)
        _lib.call("cb_elementwise", ctypes.byref(a), stream)

    def _step_reduce(self, step: Step, stream: int) -> None:
        src: View = step.args["src"]
        a = _lib.ReduceArgs()
        a.in_ = self.ptr(src)
        a.in_dtype = _lib.dtype_code(src.dtype)
        a.out = self.ptr(step.out)
        a.out_dtype = _lib.dtype_code(step.out.dtype)
        a.kind = _lib.REDUCE_SUM if step.args["how"] == "sum" else _lib.REDUCE_MAX
        a.sequential = int(step.args["sequential"])
        a.acc_dtype = _lib.dtype_code(step.out.dtype)
        keep, red = step.args["keep"], step.args["red"]
        a.n_keep, a.n_red = len(keep), len(red)
        for i, d in enumerate(keep):
            a.keep_shape[i] = src.shape[d]
            a.keep_strides[i] = src.strides[d]
        for i, d in enumerate(red):
            a.red_shape[i] = src.shape[d]
            a.red_strides[i] = src.strides[d]
        _lib.call("cb_reduce", ctypes.byref(a), stream)

    # ---------------------------------------------------- few-row matmuls
    def _rows_shape(self, step: Step):
        """(m, n, k, lda) when a MATMUL has too few rows for cb_gemm_tc: cb_gemm_rows takes it."""
        shape = gemm_shape(step, 1)
        if shape is None:
            return None
        m, n, k, lda, ldb = shape
        if m >= self._compiler.gemm_min_rows or m > 256 or ldb != k:
            return None
        return m, n, k, lda

    def _group_row_matmuls(self) -> None:
        """Group few-row matmuls that share their x into one cb_gemm_rows launch (up to 3).

        The later members run early, at the first one: their x is the same
        buffer and their weights are program inputs, and a matmul's output
        is a fresh buffer nothing reads before the matmul itself.
        """
        self._rows: Dict[int, List[Step]] = {}
        self._rows_skip: set = set()
        self._rows_counter_off: Dict[int, int] = {}
        steps = self.plan.steps
        for i, step in enumerate(steps):
            if step.name != "matmul" or id(step) in self._rows_skip:
                continue
            shape = self._rows_shape(step)
            if shape is None:
                continue
            a: View = step.args["a"]
            group = [step]
            for later in steps[i + 1:]:
                if len(group) == 3:
                    break
                if later.name != "matmul" or id(later) in self._rows_skip:
                    continue
                other = self._rows_shape(later)
                la: View = later.args["a"]
                if (other is not None and other[0] == shape[0] and other[2] == shape[2] and other[3] == shape[3]
                        and la.buf is a.buf and la.offset == a.offset and la.dtype == a.dtype
                        and later.args["b"].buf.kind == "input"):
                    group.append(later)
            self._rows[id(step)] = group
            self._rows_skip.update(id(g) for g in group[1:])

    def _rows_args(self, group: List[Step], counters: int) -> _lib.GemmRowsArgs:
        m, _, k, lda = self._rows_shape(group[0])
        a: View = group[0].args["a"]
        g = _lib.GemmRowsArgs()
        g.x = self.ptr(a) if self._built else 0
        g.x_dtype, g.ldx, g.rows, g.k, g.n_w = _lib.dtype_code(a.dtype), lda, m, k, len(group)
        for i, st in enumerate(group):
            n = st.args["b"].shape[-1]
            g.w[i] = self.ptr(st.args["b"]) if self._built else 0
            g.w_rows[i], g.ldo[i] = n, n
            g.out[i] = self.ptr(st.out) if self._built else 0
        g.splits = 0
        g.counters = counters
        return g

    def _gemm_scratch_bytes(self, step: Step) -> int:
        shape = gemm_shape(step, self._compiler.gemm_min_rows)
        if shape is None:
            return 0
        m, _, k, _, _ = shape
        # float32 A: hi and lo planes; bf16 A: one plane, used when its rows are
        # not 16-byte aligned (known only once the pointer is bound)
        return (4 if step.args["a"].dtype == np.float32 else 2) * m * k

    def _step_matmul(self, step: Step, stream: int) -> None:
        if id(step) in self._rows_skip:
            return  # launched with the first matmul of its cb_gemm_rows group
        group = self._rows.get(id(step))
        if group is not None:
            off = self._rows_counter_off[id(step)]
            g = self._rows_args(group, self._rows_counters.data_ptr() + 4 * off)
            g.scratch = self._gemm_scratch.data_ptr()
            g.error_flag = self._gemm_flag.data_ptr()
            _lib.call("cb_gemm_rows", ctypes.byref(g), stream)
            self._extra_launches += 2 - len(group)  # plane pass + GEMM for len(group) steps
            return
        av: View = step.args["a"]
        bv: View = step.args["b"]
        out = step.out
        shape = gemm_shape(step, self._compiler.gemm_min_rows)
        if shape is not None:
            m, n, k, lda, ldb = shape
            g = _lib.GemmArgs()
            g.a, g.a_dtype, g.lda = self.ptr(av), _lib.dtype_code(av.dtype), lda
            g.b, g.ldb = self.ptr(bv), ldb
            g.c, g.ldc = self.ptr(out), n
            g.m, g.n, g.k = m, n, k
            g.a_split = self._gemm_scratch.data_ptr()
            g.error_flag = self._gemm_flag.data_ptr()
            if g.b % 16 == 0 and g.c % 16 == 0:
                _lib.call("cb_gemm_tc", ctypes.byref(g), stream)
                self._extra_launches += int(av.dtype == np.float32 or g.a % 16 != 0 or lda % 8 != 0)
                return
        batch = tuple(out.shape[:-2])
        if len(batch) > _lib.MM_MAX_BATCH:
            raise _lib.KernelError("matmul: too many batch dimensions")
        a = _lib.MatmulArgs()
        a.a, a.a_dtype = self.ptr(av), _lib.dtype_code(av.dtype)
        a.b, a.b_dtype = self.ptr(bv), _lib.dtype_code(bv.dtype)
        a.c, a.c_dtype = self.ptr(out), _lib.dtype_code(out.dtype)
        a.m, a.k = av.shape[-2], av.shape[-1]
        a.n = bv.shape[-1]
        a.a_rs, a.a_cs = av.strides[-2], av.strides[-1]
        a.b_rs, a.b_cs = bv.strides[-2], bv.strides[-1]
        a.batch_ndim = len(batch)
        for d, n in enumerate(batch):
            a.batch_shape[d] = n
            for view, target in ((av, a.a_bstride), (bv, a.b_bstride)):
                j = d - (len(batch) - (len(view.shape) - 2))
                target[d] = 0 if j < 0 or view.shape[j] == 1 else view.strides[j]
        _lib.call("cb_matmul", ctypes.byref(a), stream)

    def _step_all_reduce(self, step: Step, stream: int) -> None:
        from . import parallel

        src: View = step.args["src"]
        comm = parallel.get_group(step.args["group"])
        residual: Optional[View] = step.args.get("residual")
        code = _lib.dtype_code(src.dtype)
        if residual is not None and not (comm.peer and code == _lib.F32 and src.size <= comm.peer_max_count):
            # NCCL sums into the output, then the residual is added to it in place
            comm.all_reduce(self.ptr(src), self.ptr(step.out), src.size, code, stream)
            self._add_into(step.out, residual, stream)
            return
        comm.all_reduce(self.ptr(src), self.ptr(step.out), src.size, code, stream,
                        error_flag=self.error_pointer(),
                        residual=None if residual is None else self.ptr(residual),
                        residual_dtype=_lib.F32 if residual is None else _lib.dtype_code(residual.dtype))

    def _step_all_gather(self, step: Step, stream: int) -> None:
        from . import parallel

        src: View = step.args["src"]
        comm = parallel.get_group(step.args["group"])
        if step.out.size != src.size * comm.world_size:
            raise ValueError(f"all_gather of {step.out.shape[0]} shards over a group of {comm.world_size} ranks")
        comm.all_gather(self.ptr(src), self.ptr(step.out), src.size, _lib.dtype_code(src.dtype), stream)

    def _matmul_rows_args(self, step: Step, counters: int) -> _lib.GemmRowsArgs:
        """cb_gemm_rows arguments of a planner-fused row GEMM (prologue / residual epilogue)."""
        g = step.args
        x: View = g["x"]
        a = _lib.GemmRowsArgs()
        a.x = self.ptr(x) if self._built else 0
        a.x_dtype, a.ldx, a.rows, a.k = _lib.dtype_code(x.dtype), g["ldx"], g["m"], g["k"]
        a.n_w = len(g["weights"])
        ldo = g.get("ldo") or [out.shape[-1] for out in g["outs"]]
        for i, (w, shape, out) in enumerate(zip(g["weights"], g["shapes"], g["outs"])):
            a.w[i] = self.ptr(w) if self._built else 0
            a.w_rows[i], a.ldo[i] = shape[1], ldo[i]
            a.out[i] = self.ptr(out) if self._built else 0
        a.splits, a.counters = 0, counters
        a.x_mode = g["x_mode"]
        if g["x_mode"] == _lib.ROWS_X_RMS:
            spec = g["spec"]
            w: View = g["norm_w"]
            a.norm_w = self.ptr(w) if self._built else 0
            a.norm_w_dtype = _lib.dtype_code(w.dtype)
            a.divisor, a.eps = spec.divisor, spec.eps
            (a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y) = (_lib.dtype_code(d) for d in spec.dts)
            a.dt_out = _lib.dtype_code(spec.out_dtype)
        elif g["x_mode"] == _lib.ROWS_X_SWIGLU:
            x2: View = g["x2"]
            a.x2 = self.ptr(x2) if self._built else 0
            a.x2_dtype, a.ldx2 = _lib.dtype_code(x2.dtype), x2.shape[-1]
        if g["residual"] is not None:
            r: View = g["residual"]
            a.residual = self.ptr(r) if self._built else 0
            a.ldr = r.shape[-1]
        return a

    def _step_matmul_rows(self, step: Step, stream: int) -> None:
        a = self._matmul_rows_args(step, self._rows_counters.data_ptr() + 4 * self._rows_counter_off[id(step)])
        a.scratch = self._gemm_scratch.data_ptr()
        a.error_flag = self._gemm_flag.data_ptr()
        a.pdl = int(self._compiler.pdl)
        _lib.call("cb_gemm_rows", ctypes.byref(a), stream)
        self._extra_launches += 1  # the plane pass

    @staticmethod
    def _multi_scratch_bytes(step: Step) -> int:
        g = step.args
        dt = g["spec"].out_dtype if g["x_mode"] == _lib.ROWS_X_RMS else g["a"].dtype
        return (4 if dt == np.float32 else 2) * g["m"] * g["k"]

    def _step_matmul_multi(self, step: Step, stream: int) -> None:
        """cb_gemm_tc_multi: grouped x @ W.T (q/k/v), or with a residual / SwiGLU epilogue."""
        g = step.args
        a = _lib.GemmMultiArgs()
        av: View = g["a"]
        a.a, a.a_dtype, a.lda = self.ptr(av), _lib.dtype_code(av.dtype), g["lda"]
        a.m, a.k = g["m"], g["k"]
        a.n_w = len(g["weights"])
        for i, (w, shape) in enumerate(zip(g["weights"], g["shapes"])):
            a.b[i], a.ldb[i], a.n[i] = self.ptr(w), shape[4], shape[1]
        for i, out in enumerate(g["outs"]):
            a.c[i], a.ldc[i] = self.ptr(out), out.shape[-1]
        a.epilogue = g["epilogue"]
        if g["residual"] is not None:
            r: View = g["residual"]
            a.residual, a.ldr = self.ptr(r), r.shape[-1]
        a.a_split = self._gemm_scratch.data_ptr()
        a.error_flag = self._gemm_flag.data_ptr()
        if g["x_mode"] == _lib.ROWS_X_RMS:
            spec = g["spec"]
            w: View = g["norm_w"]
            a.x_mode, a.norm_w, a.norm_w_dtype = _lib.ROWS_X_RMS, self.ptr(w), _lib.dtype_code(w.dtype)
            a.divisor, a.eps = spec.divisor, spec.eps
            (a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y) = (_lib.dtype_code(d) for d in spec.dts)
            a.dt_out = _lib.dtype_code(spec.out_dtype)
        _lib.call("cb_gemm_tc_multi", ctypes.byref(a), stream)
        direct = g["x_mode"] == _lib.ROWS_X_PLAIN and av.dtype == _BF16 and a.a % 16 == 0 and g["lda"] % 8 == 0
        self._extra_launches += int(not direct)  # the plane pass

    def _step_kv_write(self, step: Step, stream: int) -> None:
        cache: View = step.args["cache"]
        row: View = step.args["row"]
        wm: View = step.args["write_mask"]
        b, h, ctx, hd = cache.shape
        _lib.call("cb_kv_write", self.ptr(cache), b, h, ctx, hd, self.ptr(row), _lib.dtype_code(row.dtype),
                  _lib.ll_array(row.strides), self.ptr(wm), _lib.dtype_code(wm.dtype),
                  _lib.dtype_code(step.args["one_minus"]), stream)

    def _step_place(self, step: Step, stream: int) -> None:
        src: View = step.args["src"]
        cols: Buffer = step.args["cols"]
        _lib.call("cb_place_columns", self.ptr(src), _lib.dtype_code(src.dtype), len(src.shape),
                  _lib.ll_array(src.shape), _lib.ll_array(src.strides), self._ptr[cols], cols.size,
                  self.ptr(step.out), _lib.dtype_code(step.out.dtype), stream)

    def _step_gather(self, step: Step, stream: int) -> None:
        table: View = step.args["table"]
        idx: View = step.args["idx"]
        rows = table.shape[0]
        row_bytes = int(np.prod(table.shape[1:])) * table.dtype.itemsize
        _lib.call("cb_gather", self.ptr(table), rows, row_bytes, self.ptr(idx),
                  _lib.dtype_code(idx.dtype), idx.size, self.ptr(step.out),
                  self._ptr[step.args["flag"]], stream)

    def _rms_args(self, x_ptr: int, x_dtype, rows: int, width: int, spec) -> _lib.RmsNormArgs:
        a = _lib.RmsNormArgs()
        a.x, a.x_dtype = x_ptr, _lib.dtype_code(x_dtype)
        a.rows, a.width, a.x_row_stride, a.x_offset = rows, width, width, 0
        a.divisor, a.eps = spec.divisor, spec.eps
        (a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y) = (_lib.dtype_code(d) for d in spec.dts)
        return a

    def _step_rms_norm(self, step: Step, stream: int) -> None:
        x: View = step.args["x"]
        w: View = step.args["w"]
        width = x.shape[-1] if x.shape else 1
        rows = x.size // max(width, 1)
        a = self._rms_args(self.ptr(x), x.dtype, rows, width, step.args["spec"])
        a.w, a.w_dtype = self.ptr(w), _lib.dtype_code(w.dtype)
        a.out, a.out_dtype = self.ptr(step.out), _lib.dtype_code(step.out.dtype)
        _lib.call("cb_rmsnorm", ctypes.byref(a), stream)

    def _step_rope(self, step: Step, stream: int) -> None:
        x: View = step.args["x"]
        a = _lib.RopeArgs()
        a.x, a.x_dtype, a.x_offset = self.ptr(x), _lib.dtype_code(x.dtype), 0
        for d in range(4):
            a.x_strides[d] = x.strides[d]
        a.out, a.out_dtype = self.ptr(step.out), _lib.dtype_code(step.out.dtype)
        a.batch, a.heads, a.tokens, a.head_size = x.shape
        a.cos_table = self._ptr[step.args["cos"]]
        a.sin_table = self._ptr[step.args["sin"]]
        a.n_offsets = step.args["n_offsets"]
        offset = step.args["offset"]
        if offset is not None:
            a.offset, a.offset_dtype = self.ptr(offset), _lib.dtype_code(offset.dtype)
        a.error_flag = self._ptr[step.args["flag"]]
        _lib.call("cb_rope", ctypes.byref(a), stream)

    def _sdpa_tc(self, step: Step) -> bool:
        """Whether the attention runs on cb_sdpa_tc (tensor cores) rather than cb_sdpa."""
        q, k = step.args["q"], step.args["k"]
        return q.shape[-1] in (64, 128) and q.shape[2] >= self._compiler.attn_min_rows and k.shape[2] >= 1

    def _sdpa_query(self, step: Step) -> bool:
        """Whether a single-query attention (batched decode) runs on cb_sdpa_query."""
        q, k, v = step.args["q"], step.args["k"], step.args["v"]
        if q.shape[2] != 1 or q.shape[-1] not in (32, 64, 128, 256):
            return False
        for view in (k, v):
            st = [0 if n == 1 else s for n, s in zip(view.shape, view.strides)]
            if view.dtype != np.float32 or st[3] not in (0, 1) or any(x % 4 for x in st[:3]) or view.offset % 4:
                return False
        return True

    def _sdpa_scratch_bytes(self, step: Step) -> int:
        if self._sdpa_query(step):
            q, k = step.args["q"], step.args["k"]
            splits = (k.shape[2] + 31) // 32
            return q.shape[0] * q.shape[1] * splits * (q.shape[-1] + 2) * 4
        if not self._sdpa_tc(step):
            return 0
        q, k = step.args["q"], step.args["k"]
        batch, heads, tq, hd = q.shape
        kv, tk = k.shape[1], k.shape[2]
        pad = lambda t: (t + 127) // 128 * 128  # noqa: E731
        return 2 * (2 * batch * heads * pad(tq) * hd + 4 * batch * kv * pad(tk) * hd)

    def _step_sdpa(self, step: Step, stream: int) -> None:
        q, k, v, mask = (step.args[n] for n in ("q", "k", "v", "mask"))
        a = _lib.SdpaArgs()
        for name, view in (("q", q), ("k", k), ("v", v)):
            setattr(a, name, self.ptr(view))
            setattr(a, f"{name}_dtype", _lib.dtype_code(view.dtype))
            target = getattr(a, f"{name}_strides")
            for d in range(4):
                target[d] = 0 if view.shape[d] == 1 else view.strides[d]
        a.mask, a.mask_dtype = self.ptr(mask), _lib.dtype_code(mask.dtype)
        for d in range(4):
            a.mask_strides[d] = 0 if mask.shape[d] == 1 else mask.strides[d]
        a.out = self.ptr(step.out)
        if not step.out.is_contiguous():  # token-major rows (the planner's head merge without a copy)
            for d in range(4):
                a.out_strides[d] = step.out.strides[d]
        a.batch, a.heads, a.tq, a.head_size = q.shape
        a.kv_heads, a.tk = k.shape[1], k.shape[2]
        a.divisor = step.args["divisor"]
        if self._sdpa_query(step):
            _lib.call("cb_sdpa_query", ctypes.byref(a), self._gemm_scratch.data_ptr(), stream)
            self._extra_launches += 1  # the merge pass
            return
        if self._sdpa_tc(step):
            _lib.call("cb_sdpa_tc", ctypes.byref(a), int(step.args.get("causal", False)),
                      self._gemm_scratch.data_ptr(), self._gemm_flag.data_ptr(), stream)
            self._extra_launches += 1  # the plane pre-pass
            return
        _lib.call("cb_sdpa", ctypes.byref(a), stream)

    def _prefetch(self, args, target: Tuple[int, int]) -> None:
        index, cap = target
        weights: Sequence[View] = self.plan.steps[index].args["weights"]
        left = cap
        for i, w in enumerate(weights[:3]):
            size = min(w.buf.size * w.dtype.itemsize, left) & ~15
            if size <= 0:
                break
            args.prefetch_ptr[i] = self.ptr(w)
            args.prefetch_bytes[i] = size
            left -= size

    def _step_gemv(self, step: Step, stream: int) -> None:
        _lib.call("cb_gemv", ctypes.byref(self._gemv_args(step)), stream)

    def _gemv_args(self, step: Step) -> _lib.GemvArgs:
        g = step.args
        a = _lib.GemvArgs()
        weights: Sequence[View] = g["weights"]
        a.n_w = len(weights)
        for i, w in enumerate(weights):
            a.w[i] = self.ptr(w)
            a.w_rows[i] = g["rows"][i]
        a.w_dtype = _lib.dtype_code(weights[0].dtype)
        a.k = g["k"]
        x: View = g["x"]
        a.x, a.x_dtype = self.ptr(x), _lib.dtype_code(x.dtype)
        if g.get("x_index") is not None:
            a.x_index, a.x_index_dtype = self.ptr(g["x_index"]), _lib.dtype_code(g["x_index"].dtype)
            a.index_rows = x.shape[0]
        if g.get("residual_index") is not None:
            a.index_rows = g["residual"].shape[0]
        if self.plan.error_flag is not None:
            a.error_flag = self._ptr[self.plan.error_flag]
        spec = g.get("norm")
        if spec is not None:
            a.norm = _lib.NORM_RMS_TABLE if g.get("norm_table") is not None else _lib.NORM_RMS
            a.norm_w, a.norm_w_dtype = self.ptr(g["norm_w"]), _lib.dtype_code(g["norm_w"].dtype)
            a.divisor, a.eps = spec.divisor, spec.eps
            (a.dt_sq, a.dt_sum, a.dt_mean, a.dt_t, a.dt_d, a.dt_y) = (_lib.dtype_code(d) for d in spec.dts)
            a.dt_norm_out = _lib.dtype_code(spec.out_dtype)
            if g.get("norm_table") is not None:
                a.norm_table = self._ptr[g["norm_table"]]
        a.epilogue = g["epilogue"]
        if g.get("residual") is not None:
            a.residual, a.residual_dtype = self.ptr(g["residual"]), _lib.dtype_code(g["residual"].dtype)
            if g.get("residual_index") is not None:
                a.residual_index = self.ptr(g["residual_index"])
                a.residual_index_dtype = _lib.dtype_code(g["residual_index"].dtype)
        a.out = self.ptr(step.out)
        if g["epilogue"] == _lib.EPI_ARGMAX:
            a.scratch_val = self._ptr[g["scratch_val"]]
            a.scratch_idx = self._ptr[g["scratch_idx"]]
            a.counter = self._ptr[g["counter"]]
            a.argmax_out = self._ptr[g["argmax"]]
        if g.get("prefetch") is not None:
            self._prefetch(a, g["prefetch"])
        a.grid = self._compiler.gemv_grid
        a.pdl = int(self._compiler.pdl)
        return a

    def _step_decode_attention(self, step: Step, stream: int) -> None:
        _lib.call("cb_decode_attention", ctypes.byref(self._attention_args(step)), stream)

    def _attention_args(self, step: Step) -> _lib.DecodeAttentionArgs:
        g = step.args
        a = _lib.DecodeAttentionArgs()
        a.qkv = self.ptr(g["qkv"])
        a.q_off, a.k_off, a.v_off = g["q_off"], g["k_off"], g["v_off"]
        a.heads, a.kv_heads, a.head_size, a.context = g["heads"], g["kv_heads"], g["head_size"], g["context"]
        a.position, a.position_dtype = self.ptr(g["position"]), _lib.dtype_code(g["position"].dtype)
        a.cos_table, a.sin_table = self._ptr[g["cos"]], self._ptr[g["sin"]]
        a.n_positions = g["n_positions"]
        a.k_cache, a.v_cache = self.ptr(g["k_cache"]), self.ptr(g["v_cache"])
        a.kv_dtype = _lib.dtype_code(g["k_cache"].dtype)
        if g["v_cache"].dtype != g["k_cache"].dtype:
            raise TypeError("K and V caches of one attention step must have one dtype")
        a.write_mask = self.ptr(g["write_mask"])
        a.write_mask_dtype = _lib.dtype_code(g["write_mask"].dtype)
        a.one_minus_dtype = _lib.dtype_code(g["one_minus"])
        a.mask, a.mask_dtype = self.ptr(g["mask"]), _lib.dtype_code(g["mask"].dtype)
        a.divisor = g["divisor"]
        a.out = self.ptr(step.out)
        a.scratch = self._ptr[g["scratch"]]
        a.counters = self._ptr[g["counters"]]
        a.error_flag = self._ptr[g["flag"]]
        if g.get("prefetch") is not None:
            self._prefetch(a, g["prefetch"])
        a.split = 32
        a.pdl = int(self._compiler.pdl)
        return a

    def _step_decode_attention_batched(self, step: Step, stream: int) -> None:
        a = self._attention_args(step)
        _lib.call("cb_decode_attention_batched", ctypes.byref(a), step.args["batch"], step.args["qkv_stride"],
                  stream)

    # ------------------------------------------------------------ whole decode step
    def _step_table(self, flags: Optional[int] = None) -> Tuple[object, _lib.DecodeStepConfig]:
        """The prepared cb_decode_step table of the current bindings (one per key)."""
        if flags is None:
            flags = self._compiler.step_flags
        key = (getattr(self, "_last_key", ()), flags)
        entry = self._step_tables.get(key)
        if entry is not None:
            return entry
        steps = self.plan.steps
        phases = (_lib.StepPhase * len(steps))()
        for phase, step in zip(phases, steps):
            if step.name == "decode_attention":
                phase.kind = _lib.PHASE_ATTENTION
                phase.attention = self._attention_args(step)
            else:
                phase.kind = _lib.PHASE_GEMV
                phase.gemv = self._gemv_args(step)
        lib = _lib.load()
        torch = _torch()
        table = torch.empty(lib.cb_decode_step_table_bytes(len(steps)), dtype=torch.uint8,
                            device=self.device.torch_device)
        config = _lib.DecodeStepConfig()
        _lib.check(lib.cb_decode_step_prepare(phases, len(steps), table.data_ptr(), table.numel(), flags,
                                              ctypes.byref(config)), "cb_decode_step_prepare")
        if len(self._step_tables) >= 8:
            # A captured graph launches cb_decode_step with its key's table: a
            # table is freed only together with that graph (after the device
            # has finished with both), or a later run whose caches land at the
            # same addresses would replay a graph reading freed descriptors.
            old_key = next(iter(self._step_tables))
            self.device.synchronize()
            exec_ = self._graphs.pop(old_key[0], None)
            if exec_ is not None:
                lib.cb_graph_destroy(exec_)
            self._seen.pop(old_key[0], None)
            self._step_tables.pop(old_key)
        self._step_tables[key] = (table, config)
        return table, config

    def _launch_step(self, stream: int) -> None:
        table, config = self._step_table()
        _lib.call("cb_decode_step", table.data_ptr(), ctypes.byref(config), self._step_counters.data_ptr(),
                  self._step_flag.data_ptr(), stream)
        self.launches = 1

    def _reset_counters(self) -> None:
        """Zero every arrival/ticket counter after a kernel wait gave up."""
        if self.step_mode:
            self._step_counters.zero_()
        if getattr(self, "_rows_counters", None) is not None:
            self._rows_counters.zero_()
        for step in self.plan.steps:
            for name in ("counters", "counter"):
                buf = step.args.get(name)
                if buf is not None and buf in self._tensors:
                    self._tensors[buf].zero_()

    # ------------------------------------------------------------ cleanup
    def close(self) -> None:
        lib = _lib.load()
        for exec_ in self._graphs.values():
            lib.cb_graph_destroy(exec_)
        self._graphs.clear()
        if self._capture_stream is not None:
            lib.cb_stream_destroy(self._capture_stream)
            self._capture_stream = None
        if getattr(self, "_last_bound", None):  # the arrays the last run bound by pointer
            self._last_bound = [None] * len(self._last_bound)

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
