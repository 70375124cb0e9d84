"""Failure reporting on the host, without a GPU.

The reference raises explicit errors and never falls back silently
(chomikgrad/cuda_backend.py:356-371).  Kernel-side failures reach the host as
error-flag values that every bounded wait and index check stores; these
tests pin how the host turns each one into an exception, and how the
communicator layer reports a missing NCCL, bad arguments and a destroyed or
unknown group.  Nothing here launches a kernel.
"""

from __future__ import annotations

import ctypes

import pytest

from cuda_b200 import _lib, parallel


def test_every_error_flag_becomes_an_exception():
    assert isinstance(_lib.flag_error(_lib.FLAG_INDEX), IndexError)
    assert isinstance(_lib.flag_error(_lib.FLAG_POSITION), IndexError)
    assert isinstance(_lib.flag_error(_lib.FLAG_CONTEXT), IndexError)
    assert isinstance(_lib.flag_error(_lib.FLAG_NAN), ValueError)  # NumPy's choice on NaN probabilities
    for flag in (_lib.FLAG_WAIT_DATA, _lib.FLAG_WAIT_SLOT, _lib.FLAG_WAIT_DRAIN, _lib.FLAG_WAIT_PHASE):
        err = _lib.flag_error(flag)
        assert isinstance(err, _lib.KernelError) and "timed out" in str(err)
    assert isinstance(_lib.flag_error(99), _lib.KernelError)


def test_flag_values_match_the_header():
    from conftest import ROOT

    text = (ROOT / "include" / "chomik_b200.h").read_text()
    for name in ("INDEX", "POSITION", "CONTEXT", "WAIT_DATA", "WAIT_SLOT", "WAIT_DRAIN", "WAIT_PHASE", "NAN"):
        value = getattr(_lib, f"FLAG_{name}")
        assert f"CB_FLAG_{name} = {value}" in text, name


def test_missing_nccl_is_reported():
    lib = _lib.load()
    status = lib.cb_comm_load(b"/nonexistent/libnccl.so.2")
    if status == 0:
        pytest.skip("NCCL was already loaded in this process")
    assert b"libnccl" in lib.cb_last_error() or b"nonexistent" in lib.cb_last_error()
    with pytest.raises(_lib.KernelError):
        _lib.call("cb_comm_load", b"/nonexistent/libnccl.so.2")


def test_collective_arguments_are_checked_before_any_launch():
    with pytest.raises(_lib.KernelError, match="no communicator"):
        _lib.call("cb_all_reduce", None, 0, 0, 16, _lib.F32, None)
    with pytest.raises(_lib.KernelError, match="no communicator"):
        _lib.call("cb_all_gather", None, 0, 0, 16, _lib.F32, None)
    uid = (ctypes.c_char * 128)()
    handle = ctypes.c_void_p()
    with pytest.raises(_lib.KernelError, match="rank 3 of 2"):
        _lib.call("cb_comm_init", uid, 128, 2, 3, ctypes.byref(handle))
    with pytest.raises(_lib.KernelError, match="128-byte"):
        _lib.call("cb_comm_unique_id", uid, 16)


def test_unknown_and_destroyed_groups_raise():
    with pytest.raises(RuntimeError, match="init_group"):
        parallel.get_group("no-such-group")
    comm = parallel.Communicator("gone", 2, 0, 0)
    with pytest.raises(RuntimeError, match="destroyed"):
        comm.all_reduce(0, 0, 1, _lib.F32, 0)
    comm.close()  # closing twice is harmless
