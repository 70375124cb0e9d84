"""Install the unmodified reference package into ``baseline/_ref``.

The ``cuda-b200`` plugin is a chomik-grad plugin: it subclasses the
reference's ``Compiler`` / ``DeviceAdapter`` / ``CompiledProgram`` and
compiles the graphs that ``chomikgrad.llama`` builds.  Machines without a
reference checkout (the GPU boxes) import the package from ``baseline/_ref``,
which this recipe fills from a checkout with the stock installer (pure
Python; NumPy and ml_dtypes come from the environment, hence ``--no-deps``).
The checkout is copied to a temporary directory first because setuptools
writes build files next to the sources.

    python baseline/install_reference.py <path-to-chomik-grad-checkout>
"""

from __future__ import annotations

from pathlib import Path
import shutil
import subprocess
import sys
import tempfile

TARGET = Path(__file__).resolve().parent / "_ref"


def install(reference: str | Path, target: Path = TARGET) -> Path:
    reference = Path(reference)
    if not (reference / "chomikgrad" / "__init__.py").exists():
        raise FileNotFoundError(f"{reference} is not a chomik-grad checkout")
    with tempfile.TemporaryDirectory() as scratch:
        copy = Path(scratch) / "chomik-grad"
        shutil.copytree(reference, copy, ignore=shutil.ignore_patterns(".git", "*.egg-info", "build"))
        if target.exists():
            shutil.rmtree(target)
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                        "--no-deps", "--quiet", "--target", str(target), str(copy)], check=True)
    return target


if __name__ == "__main__":
    print(install(sys.argv[1]))
