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
BUILD_DIR = os.path.join(_HERE, "_build")
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
