"""``cuda-b200``: a B200-native compiler/device plugin for chomik-grad.

The plugin runs under the unmodified reference package: importing
``cuda_b200`` registers the ``cuda-b200`` compiler in ``chomikgrad``'s own
registry (``register_compiler``, chomikgrad/lazy.py:646-656) as a lazy
factory, so no GPU is touched until ``get_compiler("cuda-b200")`` first
instantiates it.  After that, the reference's graphs select it by name::

    import chomikgrad, cuda_b200  # noqa: F401
    program = chomikgrad.compile_graph(*outputs, compiler="cuda-b200",
                                       dynamic_inputs=...)

``chomikgrad`` must be importable; the plugin has no front-end of its own.
"""

from __future__ import annotations

import chomikgrad

BACKEND = "cuda-b200"


def _factory():
    from .compiler import CudaB200Compiler

    return CudaB200Compiler()


def install(chomikgrad_module=None, *, replace: bool = True) -> None:
    """(Re-)register ``cuda-b200`` in a chomikgrad module's registry (the imported one by default)."""
    module = chomikgrad if chomikgrad_module is None else chomikgrad_module
    module.register_compiler(BACKEND, _factory, replace=replace)


install()

__all__ = ["BACKEND", "install"]
