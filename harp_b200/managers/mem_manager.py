"""Memory tiers and offload (reference: managers/mem_manager.py:1-237 over the
NUMA/HBM allocator mem/custom_allocator.cpp).

Reference: two CPU tiers (DDR, on-package HBM); `use_hbm_allocator` switches
the allocator's target tier for the tensors created inside it; a pinned
"copy engine" thread moves tensors HBM -> DDR with bounded pending bytes; an
offloader turns that into saved-tensor hooks for activations.

B200 mapping: HBM = device memory, DDR = pinned host memory.
  * use_hbm_allocator(state): thread-local tier flag read by `empty()` below
    (device memory when True, pinned host memory when False);
  * CopyEngine: copies on a dedicated CUDA stream with cudaMemcpyAsync between
    device memory and pinned host buffers (page-locked, so the copy engine
    DMA runs concurrently with kernels), bounded by
    COPY_ENGINE_MAX_PENDING_BYTES of in-flight data;
  * HBMToDDROffloader: saved-tensor pack/unpack hooks that offload activations
    to pinned host memory during forward and bring them back for backward.
"""
from __future__ import annotations

import os
import queue
import threading
from contextlib import contextmanager
from typing import Dict, Optional

import torch

_tls = threading.local()


def on_hbm() -> bool:
    return getattr(_tls, "hbm", True)


def _native_ready() -> bool:
    if not torch.cuda.is_available():
        return False
    from .. import _native

    return _native.available()


@contextmanager
def use_hbm_allocator(state: bool = True):
    """state=False: cuda tensors created inside the block live in pinned,
    device-mapped host memory (the native allocator's host tier); True: the
    default device memory.  The flag is per thread, as the reference's."""
    prev = on_hbm()
    _tls.hbm = state
    try:
        if not state and _native_ready():
            from ..runtime import alloc

            with alloc.use_tier("host"):
                yield
        else:
            yield
    finally:
        _tls.hbm = prev


def empty(*shape, dtype=torch.bfloat16, device=None) -> torch.Tensor:
    """Allocate in the tier selected by use_hbm_allocator: device memory, or a
    cuda tensor in pinned host memory (host tier of the native allocator; a
    pinned CPU tensor when the library is not loaded)."""
    dev = torch.device(device) if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
    if on_hbm() or dev.type != "cuda":
        return torch.empty(*shape, dtype=dtype, device=dev)
    if _native_ready():
        from ..runtime import alloc

        with alloc.use_tier("host", dev.index):
            return torch.empty(*shape, dtype=dtype, device=dev)
    return torch.empty(*shape, dtype=dtype, pin_memory=True)


class CopyWork:
    """Completion handle of one copy."""

    def __init__(self):
        self._done_event = threading.Event()
        self._exception: Optional[BaseException] = None
        self._cuda_event = None
        self.tensor: Optional[torch.Tensor] = None
        self.nbytes = 0

    def reset(self):
        self._done_event.clear()
        self._exception = None
        self._cuda_event = None
        self.tensor = None
        self.nbytes = 0

    def mark_done(self, tensor=None):
        self.tensor = tensor
        self._done_event.set()

    def mark_failed(self, exc):
        self._exception = exc
        self._done_event.set()

    def wait(self):
        self._done_event.wait()
        if self._exception is not None:
            raise self._exception
        if self._cuda_event is not None:
            self._cuda_event.synchronize()
        return self.tensor


class CopyEngine:
    """Singleton: asynchronous device <-> pinned-host copies on a side stream."""

    _instance = None
    _lock = threading.Lock()

    def __init__(self):
        self.max_pending_bytes = int(os.environ.get("COPY_ENGINE_MAX_PENDING_BYTES", 200 * 1024 * 1024))
        self.total_size = 0
        self._cv = threading.Condition()
        self.work_pool: "queue.Queue[CopyWork]" = queue.Queue()
        self._streams: Dict[int, torch.cuda.Stream] = {}
        self._inflight = []

    @classmethod
    def get_instance(cls) -> "CopyEngine":
        if cls._instance is None:
            with cls._lock:
                if cls._instance is None:
                    cls._instance = cls()
        return cls._instance

    def _stream(self, device: torch.device) -> torch.cuda.Stream:
        s = self._streams.get(device.index)
        if s is None:
            s = torch.cuda.Stream(device=device)
            self._streams[device.index] = s
        return s

    def _get_work_handle(self) -> CopyWork:
        try:
            w = self.work_pool.get_nowait()
            w.reset()
            return w
        except queue.Empty:
            return CopyWork()

    def recycle_work_handle(self, work: CopyWork):
        work.reset()
        self.work_pool.put(work)

    def _reserve(self, nbytes):
        with self._cv:
            while self.total_size + nbytes > self.max_pending_bytes and self._inflight:
                w = self._inflight.pop(0)
                self._cv.release()
                try:
                    w.wait()
                finally:
                    self._cv.acquire()
                self.total_size -= w.nbytes
            self.total_size += nbytes

    def submit(self, src, to_host: bool = True, param=None, **_unused) -> CopyWork:
        """Copy `src` (a tensor) to pinned host memory (to_host) or back to its
        device; returns a CopyWork whose wait() gives the copy."""
        work = self._get_work_handle()
        t = src if isinstance(src, torch.Tensor) else torch.empty(0)
        if not t.is_cuda and to_host:
            work.mark_done(t)
            return work
        work.nbytes = t.numel() * t.element_size()
        self._reserve(work.nbytes)
        dev = t.device if t.is_cuda else torch.device("cuda", torch.cuda.current_device())
        s = self._stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            if to_host:
                dst = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                dst.copy_(t, non_blocking=True)
                t.record_stream(s)
            else:
                dst = torch.empty(t.shape, dtype=t.dtype, device=dev)
                dst.copy_(t, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s)
        work._cuda_event = ev
        work.mark_done(dst)
        if param is not None and to_host:
            param.grad = dst
        with self._cv:
            self._inflight.append(work)
        return work

    def wait_all(self):
        with self._cv:
            inflight, self._inflight = self._inflight, []
        for w in inflight:
            w.wait()
        with self._cv:
            self.total_size = 0

    def shutdown(self):
        self.wait_all()
        with CopyEngine._lock:
            if CopyEngine._instance is self:
                CopyEngine._instance = None


class HBMToDDROffloader:
    """torch.autograd.graph.saved_tensors_hooks(offloader.pack_hook,
    offloader.unpack_hook): activations saved for backward go to pinned host
    memory while forward runs and come back to the GPU in backward.  Tensors
    smaller than `min_bytes` stay on the device."""

    def __init__(self, min_bytes: int = 1 << 20):
        self.copy_engine = CopyEngine.get_instance()
        self.min_bytes = min_bytes

    def pack_hook(self, tensor: torch.Tensor):
        if not tensor.is_cuda or tensor.numel() * tensor.element_size() < self.min_bytes:
            return tensor
        return (tensor.device, self.copy_engine.submit(tensor, to_host=True))

    def unpack_hook(self, packed):
        if isinstance(packed, torch.Tensor):
            return packed
        dev, work = packed
        host = work.wait()
        out = host.to(dev, non_blocking=True)
        self.copy_engine.recycle_work_handle(work)
        return out

    def wait_all_copy_tasks(self):
        self.copy_engine.wait_all()

    def recycle(self, handle):
        self.copy_engine.recycle_work_handle(handle)
