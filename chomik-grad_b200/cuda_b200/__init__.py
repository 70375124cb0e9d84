"""``cuda-b200``: a B200-native compiler/device plugin for chomik-grad.

Importing the package registers the ``cuda-b200`` compiler (a lazy factory:
no GPU is touched until it is first used) in the package's mirror of
chomik-grad's plugin registry, whose front-end (``Tensor``, ``compile_graph``,
Llama builders) lives in :mod:`cuda_b200.frontend`.

To use the plugin from the original ``chomikgrad`` package instead::

    import chomikgrad, cuda_b200
    cuda_b200.install(chomikgrad)        # register_compiler("cuda-b200", ...)
    program = chomikgrad.compile_graph(*outputs, compiler="cuda-b200", ...)
"""

from __future__ import annotations

from .frontend.lazy import (
    CompiledProgram,
    Compiler,
    DeviceAdapter,
    GraphPlan,
    LazyNode,
    Op,
    get_compiler,
    register_compiler,
    set_default_compiler,
)
from .frontend.tensor import Tensor, compile_graph, no_grad, realize
from .frontend import llama
from .generation import GreedyVerification, verify_greedy_candidates

BACKEND = "cuda-b200"


def _factory():
    from .compiler import CudaB200Compiler

    return CudaB200Compiler()


register_compiler(BACKEND, _factory, replace=True)


def install(chomikgrad_module=None, *, replace: bool = True) -> None:
    """Register ``cuda-b200`` with the original chomikgrad package.

    The plugin classes are registered as virtual subclasses of chomikgrad's
    ``Compiler`` / ``DeviceAdapter`` / ``CompiledProgram`` ABCs so that
    ``get_compiler``'s ``isinstance`` check (lazy.py:674-676) accepts them.
    """
    if chomikgrad_module is None:
        import chomikgrad as chomikgrad_module  # type: ignore[no-redef]
    from .compiler import CudaB200Compiler
    from .device import CudaB200Device
    from .program import CudaB200Program

    lazy = chomikgrad_module.lazy
    lazy.Compiler.register(CudaB200Compiler)
    lazy.DeviceAdapter.register(CudaB200Device)
    lazy.CompiledProgram.register(CudaB200Program)
    chomikgrad_module.register_compiler(BACKEND, CudaB200Compiler, replace=replace)


__all__ = [
    "BACKEND", "CompiledProgram", "Compiler", "DeviceAdapter", "GraphPlan", "GreedyVerification",
    "LazyNode", "Op", "Tensor", "compile_graph", "get_compiler", "install", "llama", "no_grad",
    "realize", "register_compiler", "set_default_compiler", "verify_greedy_candidates",
]
