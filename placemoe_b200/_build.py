"""In-tree build of the native extensions.

Three extension modules are produced under ``placemoe_b200/_build/``:

* ``pm_kernels``  -- the sm_100a CUDA kernels (tcgen05 GEMMs, attention, norms,
  router, dispatch/combine, optimizer, P2P kernels) with their pybind11 bindings;
* ``pm_kernels_dbg`` -- the same kernels compiled with ``-DPLACEMOE_DEBUG_BOUNDS``:
  indices read from data (row tables, dispatch positions, peer ranks) are
  checked; a bad one records error 3 ("bounds check failed") and the access
  is skipped instead of faulting.  ``PLACEMOE_DEBUG_BOUNDS=1`` in the
  environment makes :func:`load_kernels` return this module;
* ``pm_planner``  -- the CPU C++ cores of the PlaceMoE planner (route statistics,
  mapping coordinate descent and proposals, partition exchange refinement,
  exact route replay).

Only :func:`build` compiles.  :func:`load_kernels` / :func:`load_planner` import
an already built module and never invoke the compiler, so a GPU machine that
received a pre-built tree starts without recompiling.
"""

from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
from types import ModuleType

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_CSRC = os.path.join(_PKG_DIR, "csrc")
BUILD_DIR = os.path.join(_PKG_DIR, "_build")

KERNELS_NAME = "pm_kernels"
DEBUG_KERNELS_NAME = "pm_kernels_dbg"
PLANNER_NAME = "pm_planner"
DEBUG_ENV = "PLACEMOE_DEBUG_BOUNDS"

CUDA_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def kernel_sources() -> list[str]:
    srcs = sorted(glob.glob(os.path.join(_CSRC, "kernels", "*.cu")))
    srcs += [os.path.join(_CSRC, "bindings.cpp"), os.path.join(_CSRC, "errors.cpp")]
    return srcs


def planner_sources() -> list[str]:
    return sorted(glob.glob(os.path.join(_CSRC, "planner", "*.cpp")))


def _so_path(name: str) -> str:
    return os.path.join(BUILD_DIR, name, f"{name}.so")


def build_kernels(verbose: bool = False, debug_bounds: bool = False) -> ModuleType:
    from torch.utils import cpp_extension

    name = DEBUG_KERNELS_NAME if debug_bounds else KERNELS_NAME
    defs = ["-DPLACEMOE_DEBUG_BOUNDS"] if debug_bounds else []
    out = os.path.join(BUILD_DIR, name)
    os.makedirs(out, exist_ok=True)
    return cpp_extension.load(
        name=name,
        sources=kernel_sources(),
        extra_cflags=CXX_FLAGS + defs,
        extra_cuda_cflags=CUDA_FLAGS + defs,
        extra_include_paths=[os.path.join(_CSRC), os.path.join(_CSRC, "kernels")],
        build_directory=out,
        verbose=verbose,
        with_cuda=True,
    )


def build_planner(verbose: bool = False) -> ModuleType:
    from torch.utils import cpp_extension

    out = os.path.join(BUILD_DIR, PLANNER_NAME)
    os.makedirs(out, exist_ok=True)
    return cpp_extension.load(
        name=PLANNER_NAME,
        sources=planner_sources(),
        extra_cflags=CXX_FLAGS,
        build_directory=out,
        verbose=verbose,
        with_cuda=False,
    )


def build(verbose: bool = False, debug_bounds: bool = True) -> None:
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))
    build_planner(verbose)
    build_kernels(verbose)
    if debug_bounds:
        build_kernels(verbose, debug_bounds=True)


def _import_so(name: str) -> ModuleType:
    if name in sys.modules:
        return sys.modules[name]
    path = _so_path(name)
    if not os.path.exists(path):
        raise ImportError(f"{name} is not built ({path} missing); run placemoe_b200._build.build()")
    import torch  # noqa: F401  (the extension links against libtorch)

    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_loader(name, loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    sys.modules[name] = module
    return module


def load_kernels() -> ModuleType:
    """The kernel module: the bounds-checked build when ``PLACEMOE_DEBUG_BOUNDS=1``."""
    if os.environ.get(DEBUG_ENV, "0") not in ("", "0"):
        return _import_so(DEBUG_KERNELS_NAME)
    return _import_so(KERNELS_NAME)


def load_debug_kernels() -> ModuleType:
    return _import_so(DEBUG_KERNELS_NAME)


def load_planner(auto_build: bool = True) -> ModuleType:
    try:
        return _import_so(PLANNER_NAME)
    except ImportError:
        if not auto_build:
            raise
        build_planner()
        return _import_so(PLANNER_NAME)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, debug_bounds="--no-debug" not in sys.argv)
    print("built", _so_path(KERNELS_NAME), _so_path(DEBUG_KERNELS_NAME), _so_path(PLANNER_NAME))
