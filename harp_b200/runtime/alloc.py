"""Two-tier device memory pools over the native allocator (csrc/alloc.cpp).

    from harp_b200.runtime import alloc
    with alloc.use_tier("host"):      # cuda tensors backed by pinned, mapped host memory
        buf = torch.empty(n, device="cuda")
    with alloc.use_tier("device"):    # capped HBM tier (HARP_MAX_HBM_MEMORY)
        ...
    alloc.stats("host")               # in_use, cached, peak, allocations, failures

Reference: mem/custom_allocator.cpp (DDR/HBM tiers with caps and a
thread-local tier switch).  Tiers are torch.cuda.MemPool objects built on
torch.cuda.memory.CUDAPluggableAllocator with the harp_host_* / harp_dev_*
entry points of the harp extension library; `use_tier` scopes allocations
with torch.cuda.use_mem_pool.  The managers' use_hbm_allocator(False) maps to
the host tier.
"""
from __future__ import annotations

import ctypes
from contextlib import contextmanager
from typing import Dict, Optional

import torch

from .. import _native

_pools: Dict[tuple, object] = {}
_lib: Optional[ctypes.CDLL] = None


def _so() -> str:
    _native.require()
    return _native.so_path()


def _clib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(_so())
        _lib.harp_alloc_stats.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]
        _lib.harp_alloc_set_cap.argtypes = [ctypes.c_int, ctypes.c_longlong]
    return _lib


def pool(tier: str, device: Optional[int] = None):
    """The MemPool of `tier` ("host" or "device") for `device`."""
    dev = torch.cuda.current_device() if device is None else device
    key = (tier, dev)
    if key not in _pools:
        names = {"host": ("harp_host_malloc", "harp_host_free"),
                 "device": ("harp_dev_malloc", "harp_dev_free")}[tier]
        a = torch.cuda.memory.CUDAPluggableAllocator(_so(), *names)
        with torch.cuda.device(dev):
            _pools[key] = torch.cuda.MemPool(a.allocator())
    return _pools[key]


@contextmanager
def use_tier(tier: str, device: Optional[int] = None):
    """Route this thread's cuda allocations to `tier` inside the block."""
    if tier not in ("host", "device"):
        raise ValueError(tier)
    with torch.cuda.use_mem_pool(pool(tier, device)):
        yield


def stats(tier: str) -> Dict[str, int]:
    out = (ctypes.c_longlong * 5)()
    _clib().harp_alloc_stats(0 if tier == "host" else 1, out)
    return dict(zip(("in_use", "cached", "peak", "allocations", "failures"), list(out)))


def set_cap(tier: str, nbytes: int) -> None:
    _clib().harp_alloc_set_cap(0 if tier == "host" else 1, int(nbytes))


def empty_host_cache() -> None:
    _clib().harp_host_empty_cache()
