"""Device storage and the ``DeviceAdapter`` of the ``cuda-b200`` backend.

Native values are :class:`DeviceArray` objects: a dense, C-contiguous CUDA
buffer (owned by a ``torch.Tensor``, which supplies the allocator and the
current stream) plus NumPy metadata (``shape``, ``dtype`` -- bfloat16 is
``ml_dtypes.bfloat16``), the attributes chomik-grad callers read from native
values (``Tensor.from_native(value, shape=value.shape, ...)``,
generate_tinyllama.py:796-804).

The adapter follows ``DeviceAdapter`` (chomikgrad/lazy.py:107-151):
``argmax`` has ``np.argmax`` semantics (first maximum, NaN wins) and returns
a Python int after a 8-byte read-back; there is no host fallback.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any, Dict, Mapping, Optional, Sequence

import numpy as np

from . import _lib
from chomikgrad.lazy import DeviceAdapter


def _torch():
    import torch

    return torch


def _bf16() -> np.dtype:
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


def torch_dtype(dtype: np.dtype):
    torch = _torch()
    dtype = np.dtype(dtype)
    table = {
        "float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
        "int32": torch.int32, "int64": torch.int64, "uint8": torch.uint8, "bool": torch.bool,
        "int16": torch.int16, "int8": torch.int8, "float64": torch.float64,
    }
    try:
        return table[dtype.name]
    except KeyError as error:
        raise TypeError(f"cuda-b200 cannot store dtype {dtype}") from error


def numpy_dtype(tdtype) -> np.dtype:
    torch = _torch()
    if tdtype == torch.bfloat16:
        return _bf16()
    return np.dtype(str(tdtype).replace("torch.", ""))


class DeviceArray:
    """A dense device buffer with NumPy shape/dtype metadata.

    A small host array handed to ``CudaB200Device.array`` is kept as a
    pending upload (``host``) until its device tensor is first needed: a
    program that binds it as a per-step input copies it straight into its
    own input slots (one pinned staging copy for all of a step's inputs)
    instead of through a separate device buffer.  Reading ``tensor``
    uploads it.
    """

    __slots__ = ("_tensor", "host", "device", "shape", "dtype", "argmax_value", "__weakref__")

    def __init__(self, tensor: Any, shape: Optional[Sequence[int]] = None,
                 dtype: Optional[np.dtype] = None, *, host: Optional[np.ndarray] = None,
                 device: Any = None) -> None:
        self._tensor = tensor
        self.host = host
        self.device = device
        self.shape = tuple(int(n) for n in (shape if shape is not None else tensor.shape))
        self.dtype = np.dtype(dtype) if dtype is not None else numpy_dtype(tensor.dtype)
        # Optional device int64 holding argmax(self) computed by the program
        # that produced this array (saves a reduction in DeviceAdapter.argmax).
        self.argmax_value = None

    @property
    def tensor(self) -> Any:
        if self._tensor is None:
            self._tensor = upload(self.host, self.device).tensor
            self.host = None
        return self._tensor

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    def data_ptr(self) -> int:
        return int(self.tensor.data_ptr())

    def __repr__(self) -> str:
        where = self.tensor.device if self._tensor is not None else f"{self.device} (upload pending)"
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype}, device={where})"


def empty(shape: Sequence[int], dtype: np.dtype, device: Any) -> DeviceArray:
    torch = _torch()
    count = int(np.prod(shape)) if len(shape) else 1
    tensor = torch.empty(max(count, 1), dtype=torch_dtype(dtype), device=device)
    return DeviceArray(tensor, tuple(shape), dtype)


def upload(value: np.ndarray, device: Any) -> DeviceArray:
    """Copy a host array to a new dense device buffer."""
    torch = _torch()
    host = np.asarray(value)
    shape, dtype = host.shape, host.dtype
    flat = np.ascontiguousarray(host).reshape(-1)  # (ascontiguousarray makes 0-d arrays 1-d)
    if dtype.name == "bfloat16":
        tensor = torch.from_numpy(flat.view(np.int16)).to(device).view(torch.bfloat16)
    else:
        tensor = torch.from_numpy(flat).to(device)
    if tensor.numel() == 0:
        tensor = torch.empty(1, dtype=torch_dtype(dtype), device=device)
    return DeviceArray(tensor, shape, dtype)


def download(array: DeviceArray) -> np.ndarray:
    if array.host is not None:  # never uploaded: the host copy is the value
        return np.array(array.host, copy=True).reshape(array.shape)
    torch = _torch()
    flat = array.tensor[: array.size] if array.size else array.tensor[:0]
    if array.dtype.name == "bfloat16":
        host = flat.view(torch.int16).cpu().numpy().view(np.uint16).view(_bf16())
    else:
        host = flat.cpu().numpy()
    return host.reshape(array.shape).copy()


_UPLOADABLE = frozenset(("float32", "bfloat16", "float16", "int32", "int64"))


class CudaB200Device(DeviceAdapter):
    """``DeviceAdapter`` over one B200 (the current CUDA device by default)."""

    name = "cuda-b200"
    PENDING_BYTES = 64 * 1024  # host arrays up to this size are uploaded lazily

    def __init__(self, index: Optional[int] = None) -> None:
        torch = _torch()
        if not torch.cuda.is_available():
            raise RuntimeError("the cuda-b200 backend requires a working NVIDIA driver and CUDA GPU")
        self.index = torch.cuda.current_device() if index is None else int(index)
        self.torch_device = torch.device("cuda", self.index)
        major, minor = torch.cuda.get_device_capability(self.index)
        if (major, minor) != (10, 0):
            raise RuntimeError(f"cuda-b200 kernels are built for sm_100a; device {self.index} "
                               f"is sm_{major}{minor}")
        _lib.load()
        self.sm_count = int(torch.cuda.get_device_properties(self.index).multi_processor_count)
        self.inference_dtype = _bf16()

    # -- stream ------------------------------------------------------------
    def stream(self) -> int:
        torch = _torch()
        return int(torch.cuda.current_stream(self.torch_device).cuda_stream)

    # -- DeviceAdapter -----------------------------------------------------
    def array(self, value: object) -> DeviceArray:
        if isinstance(value, DeviceArray):
            return value
        torch = _torch()
        if isinstance(value, torch.Tensor):
            tensor = value.detach().to(self.torch_device).contiguous().reshape(-1)
            return DeviceArray(tensor, tuple(value.shape), numpy_dtype(value.dtype))
        host = np.asarray(value)
        if host.nbytes <= self.PENDING_BYTES and host.dtype.name in _UPLOADABLE:
            # a small per-step input: upload when first needed (a program
            # binding it copies it into its input slots directly)
            return DeviceArray(None, host.shape, host.dtype, host=np.array(host, copy=True),
                               device=self.torch_device)
        with torch.cuda.device(self.torch_device):
            return upload(host, self.torch_device)

    def evaluate(self, values: Sequence[object]) -> None:
        self.synchronize()

    def synchronize(self) -> None:
        _torch().cuda.synchronize(self.torch_device)

    def to_numpy(self, value: object) -> np.ndarray:
        if isinstance(value, DeviceArray):
            return download(value)
        return np.asarray(value)

    def argmax(self, value: object) -> int:
        """Index of the first maximum of the flattened array (np.argmax)."""
        array = self.array(value)
        if array.argmax_value is not None:
            index, status = array.argmax_value.tolist()
            if status:  # the producing program's error flag, read with the index
                raise _lib.flag_error(int(status))
            return int(index)
        if array.size == 0:
            raise ValueError("attempt to get argmax of an empty sequence")
        result = _torch().empty(1, dtype=_torch().int64, device=self.torch_device)
        _lib.call("cb_argmax_rows", array.data_ptr(), _lib.dtype_code(array.dtype), 1,
                  array.size, result.data_ptr(), self.stream())
        return int(result.item())

    def argmax_last_axis(self, value: object) -> np.ndarray:
        array = self.array(value)
        width = array.shape[-1] if array.shape else 1
        if width == 0:
            raise ValueError("attempt to get argmax of an empty sequence")
        rows = array.size // width
        result = _torch().empty(max(rows, 1), dtype=_torch().int64, device=self.torch_device)
        if rows:
            _lib.call("cb_argmax_rows", array.data_ptr(), _lib.dtype_code(array.dtype), rows, width,
                      result.data_ptr(), self.stream())
        return result[:rows].cpu().numpy().reshape(array.shape[:-1])

    def sample(self, value: object, *, temperature: float, top_k: int, rng: np.random.Generator) -> int:
        """The reference's sampler on the device (generate_tinyllama.py:124-157).

        Samples row 0 of the logits (the reference reads ``logits[0]``):
        temperature 0 is ``argmax``; otherwise one ``rng.random()`` draw --
        the one NumPy's ``Generator.choice`` would take -- selects the token
        in cb_sample_rows, so only 8 bytes cross each way instead of the
        logit row.  Raises ValueError where NumPy's choice does (NaN
        probabilities).
        """
        if temperature == 0:
            return self.argmax(value)
        array = self.array(value)
        width = array.shape[-1] if array.shape else 1
        return int(self._sample(array, 1, width, temperature, top_k, rng)[0])

    def sample_rows(self, value: object, *, temperature: float, top_k: int,
                    rng: np.random.Generator) -> np.ndarray:
        """``sample`` for every row of the last axis, drawing in row order (batched decode)."""
        if temperature == 0:
            return self.argmax_last_axis(value)
        array = self.array(value)
        width = array.shape[-1] if array.shape else 1
        rows = array.size // width if width else 0
        return self._sample(array, rows, width, temperature, top_k, rng).reshape(array.shape[:-1])

    def _sample(self, array: DeviceArray, rows: int, width: int, temperature: float, top_k: int,
                rng: np.random.Generator) -> np.ndarray:
        if width == 0:
            raise ValueError("cannot sample from an empty sequence")
        if not np.isfinite(temperature) or temperature < 0:
            raise ValueError(f"temperature must be finite and >= 0 on cuda-b200, got {temperature}")
        torch = _torch()
        uniforms = rng.random(rows)  # the draws rng.choice would take, in row order
        dev = self.torch_device
        u = torch.from_numpy(uniforms).to(dev, non_blocking=False)
        result = torch.empty(rows + 1, dtype=torch.int64, device=dev)  # tokens, then the error flag
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        a = _lib.SampleArgs()
        a.logits, a.logits_dtype = array.data_ptr(), _lib.dtype_code(array.dtype)
        a.rows, a.width, a.ld = rows, width, width
        a.temperature, a.top_k = float(temperature), int(top_k)
        a.uniforms, a.out, a.error_flag = u.data_ptr(), result.data_ptr(), flag.data_ptr()
        _lib.call("cb_sample_rows", ctypes.byref(a), self.stream())
        result[rows:].copy_(flag)
        host = result.cpu().numpy()
        if host[rows]:
            raise _lib.flag_error(int(host[rows]))
        return host[:rows].copy()

    def dtype(self, value: object) -> np.dtype:
        if isinstance(value, DeviceArray):
            return value.dtype
        return np.asarray(value).dtype

    def load_safetensors(self, path: Path, *,
                         dtype: Optional[np.dtype] = None) -> Mapping[str, DeviceArray]:
        """Read a safetensors file straight into device buffers (casting if asked)."""
        from safetensors import safe_open

        torch = _torch()
        result: Dict[str, DeviceArray] = {}
        with safe_open(str(path), framework="pt", device="cpu") as handle:
            for key in handle.keys():
                tensor = handle.get_tensor(key)
                if dtype is not None:
                    tensor = tensor.to(torch_dtype(np.dtype(dtype)))
                result[key] = self.array(tensor)
        return result

    def reset_peak_memory(self) -> None:
        _torch().cuda.reset_peak_memory_stats(self.torch_device)

    def peak_memory_bytes(self) -> Optional[int]:
        return int(_torch().cuda.max_memory_allocated(self.torch_device))
