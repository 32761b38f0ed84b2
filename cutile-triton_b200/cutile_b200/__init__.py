"""cutile_b200 — host side of the B200 (sm_100a) kernel backend for TileTriton.

* :mod:`cutile_b200.runtime` mirrors ``TritonRun`` (triton_kernel, launch,
  flatten_args, set_target) over the C ABI of libcutile_b200.so;
* :mod:`cutile_b200.shim` mirrors ``TritonShim`` (install_shim, get_kernel);
* :mod:`cutile_b200.ops` holds typed torch-facing calls of the kernels.
"""
from . import _lib
from ._lib import B200Error
from . import runtime, shim, ops
from .runtime import (JlArray, jl, TileArray, Constant, triton_kernel, triton_kernel_candidates,
                      launch, flatten_args, set_target, code_triton)
from .shim import install_shim, get_kernel

__all__ = ["B200Error", "runtime", "shim", "ops", "JlArray", "jl", "TileArray", "Constant",
           "triton_kernel", "triton_kernel_candidates", "launch", "flatten_args", "set_target",
           "code_triton", "install_shim", "get_kernel", "library_path"]


def library_path():
    return _lib.lib_path()
