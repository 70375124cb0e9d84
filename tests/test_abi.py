"""The C ABI: the library loads, exports every declared entry point, and the
ctypes structures match the header's layout (checked by compiling a probe
with the host C compiler).  No kernel is launched."""

from __future__ import annotations

import ctypes
from pathlib import Path
import re
import shutil
import subprocess

import pytest

from conftest import ROOT
from cuda_b200 import _lib

HEADER = ROOT / "include" / "chomik_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*CB_API\s+(?:int|long long|const char\*)\s+(cb_\w+)\s*\(",
                                 text, flags=re.M)))


def test_every_declared_function_is_bound_and_exported():
    names = declared_functions()
    assert len(names) >= 20
    assert sorted(_lib.EXPORTED) == names
    lib = _lib.load()
    for name in names:
        assert hasattr(lib, name), name
    assert lib.cb_abi_version() == 1
    assert lib.cb_last_error() == b""


STRUCTS = {
    "cb_elementwise_args": _lib.ElementwiseArgs,
    "cb_reduce_args": _lib.ReduceArgs,
    "cb_matmul_args": _lib.MatmulArgs,
    "cb_rmsnorm_args": _lib.RmsNormArgs,
    "cb_rope_args": _lib.RopeArgs,
    "cb_sdpa_args": _lib.SdpaArgs,
    "cb_gemv_args": _lib.GemvArgs,
    "cb_decode_attention_args": _lib.DecodeAttentionArgs,
    "cb_gemm_args": _lib.GemmArgs,
    "cb_gemm_multi_args": _lib.GemmMultiArgs,
    "cb_gemm_rows_args": _lib.GemmRowsArgs,
    "cb_step_phase": _lib.StepPhase,
    "cb_decode_step_config": _lib.DecodeStepConfig,
    "cb_sample_args": _lib.SampleArgs,
    "cb_sgd_group": _lib.SgdGroup,
}


def test_ctypes_structures_match_the_header(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "chomik_b200.h"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in cls._fields_:
            cfield = "in" if field == "in_" else field
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {cfield}));')
    lines.append("  return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([cc, f"-I{HEADER.parent}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    for line in filter(None, out):
        cname, field, value = line.split()
        cls = STRUCTS[cname]
        actual = ctypes.sizeof(cls) if field == "size" else getattr(cls, field).offset
        assert actual == int(value), (cname, field)
