"""Completion waiting for asynchronous communication (reference:
managers/ring_attn_manager.py:6-63).

CommWork is a completion handle; CPUWaitEngine is a singleton worker thread
that waits on submitted requests - torch.distributed Work objects, CUDA events,
or any object with wait() / synchronize() - and marks their handles done, so
the submitting thread never blocks in a collective's wait.  (The reference
pins that thread to a fixed core computed from the MPI rank; here a core can
be given through HARP_WAIT_ENGINE_CORE.)
"""
from __future__ import annotations

import os
import queue
import threading
from typing import Optional


class CommWork:
    def __init__(self):
        self._done_event = threading.Event()
        self._exception: Optional[BaseException] = None
        self.work_handle = None

    def mark_done(self):
        self._done_event.set()

    def mark_failed(self, exc: BaseException):
        self._exception = exc
        self._done_event.set()

    def is_completed(self) -> bool:
        return self._done_event.is_set()

    def wait(self, timeout: Optional[float] = None) -> bool:
        ok = self._done_event.wait(timeout)
        if self._exception is not None:
            raise self._exception
        return ok


class CPUWaitEngine:
    _instance = None
    _lock = threading.Lock()

    def __init__(self):
        self.task_queue: "queue.Queue" = queue.Queue()
        self.stop_event = threading.Event()
        self.worker_thread = threading.Thread(target=self._run, name="harp-wait-engine", daemon=True)
        self.worker_thread.start()

    @classmethod
    def get_instance(cls) -> "CPUWaitEngine":
        if cls._instance is None:
            with cls._lock:
                if cls._instance is None:
                    cls._instance = cls()
        return cls._instance

    def _run(self):
        core = os.environ.get("HARP_WAIT_ENGINE_CORE")
        if core is not None and hasattr(os, "sched_setaffinity"):
            try:
                os.sched_setaffinity(threading.get_native_id(), {int(core)})
            except OSError:
                pass
        while not self.stop_event.is_set():
            try:
                req, task = self.task_queue.get(timeout=0.05)
            except queue.Empty:
                continue
            try:
                if req is not None:
                    if hasattr(req, "wait"):
                        req.wait()
                    elif hasattr(req, "synchronize"):
                        req.synchronize()
                task.mark_done()
            except BaseException as e:  # surfaced to the waiter
                task.mark_failed(e)
            finally:
                self.task_queue.task_done()

    def submit(self, req) -> CommWork:
        task = CommWork()
        task.work_handle = req
        self.task_queue.put((req, task))
        return task

    def shutdown(self):
        self.stop_event.set()
        self.worker_thread.join()
        with CPUWaitEngine._lock:
            if CPUWaitEngine._instance is self:
                CPUWaitEngine._instance = None
