"""Build and load the harp_b200 CUDA library (sm_100a).

The library is compiled in-tree into ``harp_b200/_build/harp_b200_C.so`` with
``torch.utils.cpp_extension`` and ``-gencode arch=compute_100a,code=sm_100a``.
A stamp file records a hash of every source under ``csrc/`` plus the flags;
``load()`` imports the prebuilt library when the stamp matches, so a machine
that received the built tree never recompiles.

On a machine with a GPU the kernels are the only implementation of the hot
ops: ``require()`` raises if the library cannot be loaded there, so a missing
build can never silently fall back to PyTorch ops.
"""
from __future__ import annotations

import glob
import hashlib
import os
import shutil
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(_HERE, "csrc")
# HARP_DEBUG_BOUNDS=1 selects the bounds-checking build (its own directory):
# the TMA and tcgen05 helpers check coordinates and tensor-memory columns,
# record violations (torch.ops.harp.debug_bounds_status()) and skip the access.
DEBUG_BOUNDS = os.environ.get("HARP_DEBUG_BOUNDS", "") == "1"
BUILD_DIR = os.path.join(_HERE, "_build_bounds" if DEBUG_BOUNDS else "_build")
NAME = "harp_b200_C"
SOURCES = [
    "ops.cpp",
    "gemm_sm100.cu",
    "elementwise.cu",
    "attention_sm100.cu",
    "comm.cu",
    "runtime.cpp",
    "noalloc_rmsnorm.cu",
    "alloc.cpp",
    "ulysses.cu",
    "ring.cu",
]
CUDA_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
if DEBUG_BOUNDS:
    CUDA_FLAGS = CUDA_FLAGS + ["-DHARP_DEBUG_BOUNDS"]

_lock = threading.Lock()
_loaded = False
_load_error: Exception | None = None


def so_path() -> str:
    return os.path.join(BUILD_DIR, NAME + ".so")


def _stamp_path() -> str:
    return os.path.join(BUILD_DIR, NAME + ".stamp")


def source_hash() -> str:
    h = hashlib.sha256()
    files = sorted(glob.glob(os.path.join(CSRC, "*")))
    for f in files:
        if os.path.isfile(f):
            h.update(os.path.basename(f).encode())
            with open(f, "rb") as fh:
                h.update(fh.read())
    h.update(" ".join(CUDA_FLAGS + CXX_FLAGS).encode())
    h.update(torch.__version__.encode())
    return h.hexdigest()


def is_fresh() -> bool:
    try:
        with open(_stamp_path()) as fh:
            return fh.read().strip() == source_hash() and os.path.exists(so_path())
    except OSError:
        return False


def build(verbose: bool = False) -> str:
    """Compile every CUDA/C++ source for sm_100a and load the result."""
    global _loaded
    from torch.utils.cpp_extension import load as _load

    if shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"):
        raise RuntimeError("harp_b200: nvcc not found; cannot build the CUDA library")
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    with _lock:
        _load(
            name=NAME,
            sources=srcs,
            extra_cflags=CXX_FLAGS,
            extra_cuda_cflags=CUDA_FLAGS,
            extra_include_paths=[CSRC],
            build_directory=BUILD_DIR,
            is_python_module=False,
            verbose=verbose,
        )
        with open(_stamp_path(), "w") as fh:
            fh.write(source_hash())
        _loaded = True
    return so_path()


def load(build_if_needed: bool = True) -> bool:
    """Load the library; returns True on success (never raises)."""
    global _loaded, _load_error
    if _loaded:
        return True
    try:
        if is_fresh():
            with _lock:
                if not _loaded:
                    torch.ops.load_library(so_path())
                    _loaded = True
            return True
        if build_if_needed:
            build()
            return True
        if os.path.exists(so_path()):
            # Stale stamp but a library exists (e.g. sources edited without a
            # rebuild): load it rather than run nothing; build() refreshes it.
            with _lock:
                if not _loaded:
                    torch.ops.load_library(so_path())
                    _loaded = True
            return True
        _load_error = RuntimeError("harp_b200 CUDA library not built (run harp_b200._native.build())")
    except Exception as e:  # pragma: no cover - reported through require()
        _load_error = e
    return False


def available() -> bool:
    return _loaded or load(build_if_needed=False)


def require() -> None:
    """Raise unless the CUDA library is loaded (used by every GPU code path)."""
    if not available():
        raise RuntimeError(
            "harp_b200: CUDA kernels are required on GPU tensors but the library is not loaded: "
            f"{_load_error!r}"
        )


# ---------------------------------------------------------------------------
# the harp_nvl torch.distributed backend: a separate Python extension module
# (it needs pybind11 and the c10d headers; the op library above does not)
# ---------------------------------------------------------------------------
C10D_NAME = "harp_b200_c10d"
C10D_SOURCES = ["c10d_nvl.cpp", "c10d_nvl_kernels.cu"]
_c10d_mod = None


def c10d_so_path() -> str:
    return os.path.join(BUILD_DIR, C10D_NAME + ".so")


def _c10d_hash() -> str:
    h = hashlib.sha256()
    for s in C10D_SOURCES + ["c10d_nvl_kernels.h", "common.cuh"]:
        with open(os.path.join(CSRC, s), "rb") as fh:
            h.update(s.encode())
            h.update(fh.read())
    h.update(" ".join(CUDA_FLAGS + CXX_FLAGS).encode())
    h.update(torch.__version__.encode())
    return h.hexdigest()


def build_c10d(verbose: bool = False):
    """Compile the harp_nvl backend module for sm_100a and import it."""
    global _c10d_mod
    from torch.utils.cpp_extension import load as _load

    os.makedirs(BUILD_DIR, exist_ok=True)
    with _lock:
        _c10d_mod = _load(name=C10D_NAME, sources=[os.path.join(CSRC, s) for s in C10D_SOURCES],
                          extra_cflags=CXX_FLAGS,
                          extra_cuda_cflags=[f for f in CUDA_FLAGS if f != "-DHARP_DEBUG_BOUNDS"],
                          extra_include_paths=[CSRC],
                          build_directory=BUILD_DIR, is_python_module=True, verbose=verbose)
        with open(os.path.join(BUILD_DIR, C10D_NAME + ".stamp"), "w") as fh:
            fh.write(_c10d_hash())
    return _c10d_mod


def load_c10d(build_if_needed: bool = True):
    """The harp_nvl backend module (prebuilt in-tree, else compiled now)."""
    global _c10d_mod
    if _c10d_mod is not None:
        return _c10d_mod
    try:
        with open(os.path.join(BUILD_DIR, C10D_NAME + ".stamp")) as fh:
            fresh = fh.read().strip() == _c10d_hash() and os.path.exists(c10d_so_path())
    except OSError:
        fresh = False
    if fresh:
        import importlib.machinery
        import importlib.util

        import torch.distributed  # noqa: F401  (registers the c10d Python types the module returns)

        loader = importlib.machinery.ExtensionFileLoader(C10D_NAME, c10d_so_path())
        spec = importlib.util.spec_from_file_location(C10D_NAME, c10d_so_path(), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _c10d_mod = mod
        return mod
    if not build_if_needed:
        raise RuntimeError("harp_nvl backend module not built (run harp_b200._native.build_c10d())")
    return build_c10d()
