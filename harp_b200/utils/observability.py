"""Logging, per-phase device timing, NVTX ranges and the torch profiler
(reference: train.py:56-94 logging, :422-441 profiler, :489-537 per-phase
prints; async_rt/cpp_async_runtime.cpp RECORD_FUNCTION for native ops).

  setup_logger(log_file, is_main)  INFO on rank 0 (stream + train.log), ERROR elsewhere
  PhaseTimer                       CUDA-event timing of named phases per step,
                                   reported as the max over ranks (JSONL)
  phase(name) / enable_phases()    process-wide phase timer that the trainer
                                   and the NVLink exchanges report into (off
                                   unless enabled or HARP_PHASES=1)
  nvtx(name)                       NVTX range context manager (no-op on CPU)
  make_profiler(out_dir)           torch.profiler with CPU+CUDA activities,
                                   schedule(wait=0, warmup=2, active=4)
"""
from __future__ import annotations

import json
import logging
import os
import time
from contextlib import contextmanager
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

logger = logging.getLogger("harp_b200")


def setup_logger(log_file: Optional[str], is_main_process: bool) -> logging.Logger:
    level = logging.INFO if is_main_process else logging.ERROR
    logger.setLevel(level)
    logger.propagate = False
    for h in list(logger.handlers):
        logger.removeHandler(h)
        h.close()
    fmt = logging.Formatter("%(asctime)s - %(levelname)s - %(name)s - %(message)s", "%m/%d/%Y %H:%M:%S")
    sh = logging.StreamHandler()
    sh.setLevel(level)
    sh.setFormatter(fmt)
    logger.addHandler(sh)
    if is_main_process and log_file:
        os.makedirs(os.path.dirname(os.path.abspath(log_file)), exist_ok=True)
        fh = logging.FileHandler(log_file, mode="a", encoding="utf-8")
        fh.setLevel(level)
        fh.setFormatter(fmt)
        logger.addHandler(fh)
    return logger


@contextmanager
def nvtx(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class PhaseTimer:
    """Device time of named phases (CUDA events on the current stream); CPU
    wall-clock when no GPU.  `report()` syncs and returns max-over-ranks ms."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._marks: List = []
        self._cuda = torch.cuda.is_available()

    @contextmanager
    def phase(self, name: str):
        if not self.enabled:
            yield
            return
        with nvtx(name):
            if self._cuda:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                yield
                b.record()
                self._marks.append((name, a, b))
            else:
                t0 = time.perf_counter()
                yield
                self._marks.append((name, t0, time.perf_counter()))

    def report(self) -> Dict[str, float]:
        out: Dict[str, float] = {}
        if self._cuda:
            torch.cuda.synchronize()
        for name, a, b in self._marks:
            ms = a.elapsed_time(b) if self._cuda else (b - a) * 1e3
            out[name] = out.get(name, 0.0) + ms
        self._marks = []
        if dist.is_available() and dist.is_initialized() and out:
            keys = sorted(out)
            dev = torch.device("cuda", torch.cuda.current_device()) if self._cuda else torch.device("cpu")
            t = torch.tensor([out[k] for k in keys], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out = dict(zip(keys, t.tolist()))
        return out


_PHASES: Optional[PhaseTimer] = PhaseTimer() if os.environ.get("HARP_PHASES", "") == "1" else None


def enable_phases(on: bool = True) -> Optional[PhaseTimer]:
    """Switch the process-wide phase timer on (or off); returns it."""
    global _PHASES
    _PHASES = PhaseTimer() if on else None
    return _PHASES


def phase_timer() -> Optional[PhaseTimer]:
    return _PHASES


@contextmanager
def phase(name: str):
    """Time a named phase on the current stream when the process-wide timer
    is on; otherwise a no-op that costs one attribute lookup."""
    t = _PHASES
    if t is None:
        yield
        return
    with t.phase(name):
        yield


class JsonlWriter:
    def __init__(self, path: Optional[str]):
        self.path = path
        if path:
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)

    def write(self, rec: dict):
        if self.path:
            with open(self.path, "a") as fh:
                fh.write(json.dumps(rec) + "\n")


def make_profiler(out_dir: str, wait: int = 0, warmup: int = 2, active: int = 4):
    import torch.profiler as prof

    acts = [prof.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(prof.ProfilerActivity.CUDA)
    os.makedirs(out_dir, exist_ok=True)
    return prof.profile(activities=acts, schedule=prof.schedule(wait=wait, warmup=warmup, active=active, repeat=1),
                        on_trace_ready=prof.tensorboard_trace_handler(out_dir), record_shapes=True,
                        profile_memory=True, with_stack=True)
