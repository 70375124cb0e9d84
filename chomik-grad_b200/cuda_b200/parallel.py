"""Tensor-parallel communicators of the ``cuda-b200`` plugin.

The reference runs on one device and has no collectives.  Its Llama graphs
become tensor-parallel here (``cuda_b200.tensor_parallel``) by sharding the
heads and the MLP's intermediate dimension over the ranks of a group and
summing the row-sharded O and down projections with an all-reduce.  That
all-reduce is a step of the compiled program: ``cb_all_reduce`` (NCCL, loaded
by the kernel library) issued on the program's stream, so the CUDA graph of a
decode step replays it together with the kernels.

A group is created once per process, collectively, over an initialised
``torch.distributed`` process group (any backend: only NCCL's 128-byte unique
id travels through it), and is looked up by name when a program runs.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional

from . import _lib

_GROUPS: Dict[str, "Communicator"] = {}


def nccl_library() -> Optional[str]:
    """Path of the NCCL that ships with torch (the one torch.distributed loads), if present."""
    try:
        import nvidia.nccl  # type: ignore

        for root in nvidia.nccl.__path__:
            path = os.path.join(root, "lib", "libnccl.so.2")
            if os.path.exists(path):
                return path
    except Exception:
        pass
    return None


class Communicator:
    """One rank's NCCL communicator of a tensor-parallel group."""

    def __init__(self, name: str, world_size: int, rank: int, handle: int) -> None:
        self.name = name
        self.world_size = world_size
        self.rank = rank
        self._handle = handle

    @property
    def handle(self) -> int:
        if not self._handle:
            raise RuntimeError(f"tensor-parallel group {self.name!r} has been destroyed")
        return self._handle

    def all_reduce(self, src: int, dst: int, count: int, dtype_code: int, stream: int) -> None:
        """dst = sum over ranks of src (device pointers), issued on ``stream``."""
        _lib.call("cb_all_reduce", self.handle, src, dst, count, dtype_code, stream)

    def all_gather(self, src: int, dst: int, count: int, dtype_code: int, stream: int) -> None:
        """dst = every rank's ``count``-element src, rank after rank (device pointers), on ``stream``."""
        _lib.call("cb_all_gather", self.handle, src, dst, count, dtype_code, stream)

    def close(self) -> None:
        if self._handle:
            _lib.call("cb_comm_destroy", self._handle)
            self._handle = 0


def _load() -> None:
    path = nccl_library()
    _lib.call("cb_comm_load", path.encode() if path else None)


def init_group(name: str = "tp", process_group=None) -> Communicator:
    """Create the named group over the ranks of a ``torch.distributed`` group (collective).

    The current CUDA device must be this rank's GPU.
    """
    import torch.distributed as dist

    if name in _GROUPS:
        raise ValueError(f"tensor-parallel group {name!r} already exists")
    world = dist.get_world_size(process_group)
    rank = dist.get_rank(process_group)
    _load()
    uid = (ctypes.c_char * 128)()
    if rank == 0:
        _lib.call("cb_comm_unique_id", uid, 128)
    box = [bytes(uid)]
    src = 0 if process_group is None else dist.get_global_rank(process_group, 0)
    dist.broadcast_object_list(box, src=src, group=process_group)
    uid = (ctypes.c_char * 128).from_buffer_copy(box[0])
    handle = ctypes.c_void_p()
    _lib.call("cb_comm_init", uid, 128, world, rank, ctypes.byref(handle))
    comm = Communicator(name, world, rank, int(handle.value or 0))
    _GROUPS[name] = comm
    return comm


def get_group(name: str) -> Communicator:
    try:
        return _GROUPS[name]
    except KeyError:
        raise RuntimeError(f"no tensor-parallel group {name!r}: call cuda_b200.parallel.init_group first") from None


def destroy_group(name: str) -> None:
    """Destroy the named group's communicator (collective).

    Every CUDA graph that captured one of its all-reduces must be released
    first (``TensorParallelRuntime.close``): NCCL waits for them.
    """
    comm = _GROUPS.pop(name, None)
    if comm is not None:
        comm.close()
