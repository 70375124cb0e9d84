"""Test configuration.

``-m "not gpu"`` runs on any machine (oracle vs golden fixtures, planning,
C-ABI loading).  ``-m gpu`` tests need a B200 and call the kernels through the
C ABI; they compare against the parity oracle (``oracle/``) and the golden
fixtures made from the reference by ``tests/golden/make_golden.py``.
"""

from __future__ import annotations

import os
from pathlib import Path
import sys

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
# The plugin runs under the unmodified reference package; machines without a
# reference checkout import it from baseline/_ref (baseline/install_reference.py).
for path in (ROOT / "baseline" / "_ref", ROOT / "chomik-grad_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

# A reference checkout (its examples/ and tests/ are not in the installed
# package), only when CHOMIK_REFERENCE names one; tests that need it skip
# otherwise.  GPU tests never need it.
REFERENCE = Path(os.environ["CHOMIK_REFERENCE"]) if os.environ.get("CHOMIK_REFERENCE") else None


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA kernels)")


def golden(name: str) -> dict:
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {path.name} has not been generated")
    with np.load(path) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def oracle():
    """The restated reference ``cpu`` compiler, registered as ``cpu`` in chomikgrad's registry."""
    from oracle import numpy_compiler

    numpy_compiler.install()
    return numpy_compiler


@pytest.fixture(scope="session")
def gpu():
    """The ``cuda-b200`` compiler on cuda:0 (GPU tests only)."""
    import chomikgrad
    import cuda_b200

    return chomikgrad.get_compiler(cuda_b200.BACKEND)
