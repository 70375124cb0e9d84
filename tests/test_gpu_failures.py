"""Failure reporting on the GPU: a bounded wait of the decode step runs out on purpose.

cb_decode_step's blocks wait for one another at every phase boundary on a
grid-wide counter, each wait bounded (about 1 s).  The test knob
``cb_decode_step_config.test_withhold`` makes one block skip its arrival
after the first phase -- an arrival nothing else will make -- so every
block's next wait runs out.  The step must then stop, report
CB_FLAG_WAIT_PHASE through the error flag (raised by the program as a
KernelError), leave the context usable, and after the counters are zeroed
give the same logits as before.  No fault, no unbounded wait.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from cuda_b200.models import WORKLOADS, synthetic_weights
from cuda_b200.runtime import LlamaRuntime

pytestmark = pytest.mark.gpu


def test_decode_step_reports_a_phase_wait_that_ran_out(gpu):
    import torch

    from cuda_b200 import _lib

    wl = WORKLOADS["tiny-bf16"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200")
    prompt, context = [5, 17, 3, 99, 42, 7], 32
    logits, caches = rt.prefill(prompt, context)
    token, position = rt.device.argmax(logits), len(prompt)
    logits, caches = rt.decode(token, position, context, caches)
    want = rt.device.to_numpy(logits).copy()
    program, _ = rt.decode_program(context, caches, token, position)
    assert program.step_mode
    table, config = program._step_table()
    broken = _lib.DecodeStepConfig()
    for name, _ in _lib.DecodeStepConfig._fields_:
        setattr(broken, name, getattr(config, name))
    broken.test_withhold = 1 + 3  # block 3 withholds its arrival after phase 0
    started = time.perf_counter()
    _lib.call("cb_decode_step", table.data_ptr(), ctypes.byref(broken), program._step_counters.data_ptr(),
              program._step_flag.data_ptr(), rt.device.stream())
    torch.cuda.synchronize()
    assert time.perf_counter() - started < 30
    assert int(program._step_flag[0].item()) == _lib.FLAG_WAIT_PHASE
    with pytest.raises(_lib.KernelError, match="previous phase of the decode step"):
        program.check_errors()  # also zeroes the flag and the counters
    assert not program._step_counters.any().item()
    # the context is usable and the step gives the same logits again
    logits, caches = rt.decode(token, position, context, caches)
    np.testing.assert_array_equal(rt.device.to_numpy(logits), want)
