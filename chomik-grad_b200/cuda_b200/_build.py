"""Build ``libchomik_b200.so`` (sm_100a) in-tree with nvcc.

    python -m cuda_b200._build        # from chomik-grad_b200/

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (rebuilt only
when it or a header is newer) and linked into ``cuda_b200/libchomik_b200.so``.
Numerics rely on IEEE division/sqrt, so no fast-math flags are used.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
import os
from pathlib import Path
import shutil
import subprocess
from typing import List

PACKAGE = Path(__file__).resolve().parent
PROJECT = PACKAGE.parent
CSRC = PROJECT / "csrc"
INCLUDE = PROJECT.parent / "include"
BUILD = PROJECT / "_build"
LIBRARY = PACKAGE / "libchomik_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the cuda-b200 kernels need the CUDA toolkit")
    return found


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(source: Path, verbose: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(source.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(source), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{done.stdout}\n{done.stderr}")
    if verbose and done.stderr.strip():
        print(done.stderr, flush=True)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every kernel source and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if force:
        for obj in BUILD.glob("*.o"):
            obj.unlink()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects: List[Path] = list(pool.map(lambda s: _compile(s, verbose), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= newest and not force:
        return LIBRARY
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"link failed:\n{done.stdout}\n{done.stderr}")
    return LIBRARY


if __name__ == "__main__":
    import sys

    print(build(verbose=True, force="--force" in sys.argv))
