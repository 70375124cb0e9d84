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
id and the peer regions' 64-byte IPC handles travel through it), and is
looked up by name when a program runs.

With more than one rank a group also maps the other ranks' exchange regions
(``cb_peer_*``, CUDA IPC over NVLink): an all-reduce of at most
``PEER_MAX_COUNT`` float32 values -- the per-layer sums of the decode -- runs
as one kernel that stores this rank's partial into every rank's region and
sums the ranks' partials in rank order (``cb_peer_all_reduce``); larger ones
(the prefill's) and bfloat16 ones go to NCCL.  ``CUDA_B200_PEER_ALLREDUCE=0``
keeps every all-reduce on NCCL.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional

from . import _lib

_GROUPS: Dict[str, "Communicator"] = {}
PEER_MAX_COUNT = 1 << 20  # float32 values of the largest peer all-reduce (4 MiB per rank and buffer)


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

    def __init__(self, name: str, world_size: int, rank: int, handle: int, peer: int = 0) -> None:
        self.name = name
        self.world_size = world_size
        self.rank = rank
        self._handle = handle
        self._peer = peer  # cb_peer group (0: none)
        self.peer_max_count = PEER_MAX_COUNT if peer else 0

    @property
    def handle(self) -> int:
        if not self._handle:
            raise RuntimeError(f"tensor-parallel group {self.name!r} has been destroyed")
        return self._handle

    @property
    def peer(self) -> bool:
        return bool(self._peer)

    def all_reduce(self, src: int, dst: int, count: int, dtype_code: int, stream: int, *,
                   error_flag: Optional[int] = None, residual: Optional[int] = None,
                   residual_dtype: int = _lib.F32) -> None:
        """dst = (residual +) sum over ranks of src (device pointers), issued on ``stream``.

        The peer kernel when the group has one and the message is float32 and small enough
        (``error_flag``: where a wait that runs out is reported); NCCL otherwise."""
        if self._peer and dtype_code == _lib.F32 and count <= self.peer_max_count:
            _lib.call("cb_peer_all_reduce", self._peer, src, dst, _lib.F32, residual, residual_dtype, count,
                      error_flag, stream)
            return
        _lib.call("cb_all_reduce", self.handle, src, dst, count, dtype_code, stream)
        if residual is not None:
            raise ValueError("a residual rides along with the peer all-reduce only")

    def set_peer_wait(self, seconds: float) -> None:
        """Bound of the peer all-reduce's wait for the other ranks (tests shorten it)."""
        if self._peer:
            _lib.call("cb_peer_set_wait", self._peer, int(seconds * 1e9))

    def all_gather(self, src: int, dst: int, count: int, dtype_code: int, stream: int) -> None:
        """dst = every rank's ``count``-element src, rank after rank (device pointers), on ``stream``."""
        _lib.call("cb_all_gather", self.handle, src, dst, count, dtype_code, stream)

    def close(self) -> None:
        if self._peer:
            _lib.call("cb_peer_destroy", self._peer)
            self._peer = 0
        if self._handle:
            _lib.call("cb_comm_destroy", self._handle)
            self._handle = 0


def _load() -> None:
    path = nccl_library()
    _lib.call("cb_comm_load", path.encode() if path else None)


def init_group(name: str = "tp", process_group=None, *, peer: Optional[bool] = None) -> Communicator:
    """Create the named group over the ranks of a ``torch.distributed`` group (collective).

    The current CUDA device must be this rank's GPU.  ``peer`` (default: more
    than one rank and ``CUDA_B200_PEER_ALLREDUCE`` not "0") maps the ranks'
    exchange regions for the peer all-reduce.
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
    if peer is None:
        peer = world > 1 and os.environ.get("CUDA_B200_PEER_ALLREDUCE", "1") != "0"
    group = 0
    if peer:
        group = _connect_peers(world, rank, process_group)
    comm = Communicator(name, world, rank, int(handle.value or 0), group)
    _GROUPS[name] = comm
    return comm


def _connect_peers(world: int, rank: int, process_group) -> int:
    """Create this rank's exchange region, share its IPC handle, map the others' (collective)."""
    import torch.distributed as dist

    group = ctypes.c_void_p()
    handle = (ctypes.c_char * 64)()
    _lib.call("cb_peer_create", world, rank, PEER_MAX_COUNT, ctypes.byref(group), handle, 64)
    handles = [None] * world
    try:
        dist.all_gather_object(handles, bytes(handle), group=process_group)
        packed = (ctypes.c_char * (64 * world)).from_buffer_copy(b"".join(handles))
        _lib.call("cb_peer_connect", group, packed, 64)
    except Exception:
        _lib.call("cb_peer_destroy", group)
        raise
    dist.barrier(group=process_group)  # every rank mapped every region before any all-reduce
    return int(group.value or 0)


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
    if comm is None:
        return
    if comm.peer:
        # the other ranks' kernels may still store into this rank's region until they finish
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier()
    comm.close()
