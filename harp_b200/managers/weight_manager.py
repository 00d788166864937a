"""Parameter placement, ownership and sharded-optimizer plumbing (reference:
managers/weight_manager.py:8-221).

Reference design: the SP ranks of a CPU die share ONE copy of the weights and
gradients in POSIX shared memory; each parameter has an owner rank chosen by
balancing bytes; owners row-split their parameters over the "RS" group for
the optimizer and all-gather the updated chunks back, raising a per-parameter
ready byte that the next forward spins on.

B200 design, same API:
  * CPU tensors (gloo ranks on one host): exactly the reference scheme, POSIX
    shared memory per SP group.
  * CUDA tensors: every GPU keeps its own replica in HBM (reading weights over
    NVLink every layer would cost more than replicating them).
    `p.shared_grad` is a view into one flat device gradient buffer, `p.state`
    is a one-byte device flag, and the asynchronous all-gather runs on a side
    CUDA stream; readiness is a CUDA event the consuming stream waits on,
    instead of a host spin loop.
"""
from __future__ import annotations

import os
import queue
import threading
import time
from multiprocessing import shared_memory
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..parallel import collectives as C


def is_norm_param(name: str) -> bool:
    return "norm" in name.lower()


def is_no_shard_param(name: str) -> bool:
    return False


def _job_tag() -> str:
    for k in ("HARP_JOB_ID", "TORCH_SHM_ID", "SLURM_JOB_ID", "TORCHELASTIC_RUN_ID"):
        if os.environ.get(k):
            return os.environ[k]
    return "0"


def get_shm(shm_name: str, size: int, local_rank: int, master_rank: int, group=None):
    """Named POSIX shared-memory segment shared by the ranks of `group` on one
    host: `master_rank` creates it (replacing a stale one), the others attach."""
    shm = None
    if local_rank == master_rank:
        try:
            shm = shared_memory.SharedMemory(name=shm_name, create=True, size=max(1, size))
        except FileExistsError:
            old = shared_memory.SharedMemory(name=shm_name, create=False)
            old.close()
            old.unlink()
            shm = shared_memory.SharedMemory(name=shm_name, create=True, size=max(1, size))
    if dist.is_initialized():
        dist.barrier(group=group)
    if shm is None:
        shm = shared_memory.SharedMemory(name=shm_name, create=False)
    return shm


def setup_shared_model(model, param_rank: Dict[int, int], rank: int, local_rank: int, master_rank: int = 3,
                       grad_master_rank: int = 2, sp_size: int = 4, group=None):
    """Give every parameter `shared_grad` and `state`; on CPU also move its data
    into die-shared memory.  Returns (param store, grad store, state store)."""
    params = list(model.named_parameters())
    if not params:
        return None, None, None
    dev = params[0][1].device
    offsets, off = [], 0
    for _, p in params:
        offsets.append(off)
        off += p.numel() * p.element_size()
    total = off
    if dev.type == "cuda":
        flat_grad = torch.zeros(total, dtype=torch.uint8, device=dev)
        flat_state = torch.ones(len(params), dtype=torch.uint8, device=dev)
        for i, (name, p) in enumerate(params):
            p.shared_grad = flat_grad[offsets[i]:offsets[i] + p.numel() * p.element_size()].view(p.dtype).view(
                p.shape)
            p.state = flat_state[i]
        return None, flat_grad, flat_state
    die = rank // sp_size
    tag = _job_tag()
    master_rank = master_rank % sp_size
    grad_master_rank = grad_master_rank % sp_size
    shm = get_shm(f"harp_model_{tag}_{die}", total, local_rank, master_rank, group)
    shm_grad = get_shm(f"harp_grad_{tag}_{die}", total, local_rank, grad_master_rank, group)
    shm_state = get_shm(f"harp_state_{tag}_{die}", len(params), local_rank, master_rank, group)
    if local_rank == master_rank:
        shm_state.buf[: len(params)] = bytes(len(params))
    if dist.is_initialized():
        dist.barrier(group=group)
    states = torch.frombuffer(shm_state.buf, dtype=torch.uint8, count=len(params))
    for i, (name, p) in enumerate(params):
        n = p.numel()
        g = torch.frombuffer(shm_grad.buf, dtype=p.dtype, count=n, offset=offsets[i]).view(p.shape)
        p.shared_grad = g.detach()
        if param_rank.get(id(p)) == local_rank:
            p.shared_grad.zero_()
        if is_norm_param(name):
            p.state = torch.ones((), dtype=torch.uint8)
            continue
        p.state = states[i]
        view = torch.frombuffer(shm.buf, dtype=p.dtype, count=n, offset=offsets[i]).view(p.shape)
        if param_rank.get(id(p)) == local_rank:
            view.copy_(p.data)
        p.data = view
    if dist.is_initialized():
        dist.barrier(group=group)
    for i, (name, p) in enumerate(params):
        if not is_norm_param(name):
            p.state.fill_(1)
    return shm, shm_grad, shm_state


def build_balanced_param_groups(model, sp_size: int, local_rank: int, block_size: int = 100 * 1024 * 1024):
    """Owner rank of every parameter: norm weights round-robin by count; the
    other trainable parameters in registration order, moving to the next rank
    once the current one holds more than `block_size` bytes.  Returns
    (parameters this rank optimizes, {id(param): owner rank})."""
    param_rank: Dict[int, int] = {}
    norms = [(n, p) for n, p in model.named_parameters() if is_norm_param(n)]
    for i, (_, p) in enumerate(norms):
        param_rank[id(p)] = i % sp_size
    rank_bytes = [0] * sp_size
    cur = 0
    for name, p in model.named_parameters():
        if is_norm_param(name) or not p.requires_grad:
            continue
        if rank_bytes[cur] > 0 and rank_bytes[cur] > block_size:
            cur = (cur + 1) % sp_size
            rank_bytes[cur] = 0
        param_rank[id(p)] = cur
        rank_bytes[cur] += p.numel() * p.element_size()
    my_params = [p for n, p in model.named_parameters()
                 if p.requires_grad and (is_norm_param(n) or param_rank.get(id(p)) == local_rank)]
    return my_params, param_rank


def build_chunk_param(my_params, model, rs_size: int, rs_rank: int) -> List[torch.Tensor]:
    """Row-chunk each owned parameter over the RS group: the optimizer steps
    `p.chunk_part` (rows [chunk_begin, chunk_end)), whose `.grad` is a view of
    `p.shared_grad`.  Parameters that do not split evenly stay whole.
    Membership in `my_params` is by identity (the reference's `p in my_params`
    compares tensors by value, which raises once two parameters of different
    shapes are compared)."""
    mine = {id(p) for p in my_params}
    out = []
    for name, p in model.named_parameters():
        if id(p) not in mine:
            continue
        if p.ndim == 0 or p.shape[0] % rs_size != 0 or is_no_shard_param(name):
            out.append(p)
            continue
        chunk = p.shape[0] // rs_size
        b, e = rs_rank * chunk, (rs_rank + 1) * chunk
        part = p.detach().narrow(0, b, chunk).clone()
        part.chunk_begin, part.chunk_end = b, e
        part.requires_grad_(True)
        if hasattr(p, "shared_grad"):
            part.grad = p.shared_grad[b:e]
        p.chunk_part = part
        out.append(part)
    return out


class AsyncParamAllGatherManager:
    """All-gathers updated row chunks back into full parameters in the background
    and marks each parameter ready.  CUDA: on a side stream, readiness = an
    event (`p._harp_ready_event`) plus the device flag; CPU: a worker thread."""

    def __init__(self, rs_group, rs_size: int, core_id: Optional[int] = None):
        self.rs_group, self.rs_size, self.core_id = rs_group, rs_size, core_id
        self.exc: Optional[BaseException] = None
        self._stream = None
        self.task_queue: "queue.Queue" = queue.Queue()
        self.worker = threading.Thread(target=self._run, name="harp-param-allgather", daemon=True)
        self.worker.start()

    def push(self, p):
        if self.exc is not None:
            raise self.exc
        if p.is_cuda:
            self._gather_cuda(p)
        else:
            self.task_queue.put(p)

    def _gather_cuda(self, p):
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=p.device)
        cur = torch.cuda.current_stream(p.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self._all_gather(p)
            ev = torch.cuda.Event()
            ev.record(self._stream)
            p._harp_ready_event = ev

    def wait_all(self):
        self.task_queue.join()
        if self._stream is not None:
            torch.cuda.current_stream(self._stream.device).wait_stream(self._stream)
        if self.exc is not None:
            raise self.exc

    def shutdown(self):
        self.task_queue.put(None)
        self.worker.join()
        if self.exc is not None:
            raise self.exc

    def _run(self):
        if self.core_id is not None and hasattr(os, "sched_setaffinity"):
            try:
                os.sched_setaffinity(threading.get_native_id(), {self.core_id})
            except OSError:
                pass
        while True:
            p = self.task_queue.get()
            try:
                if p is None:
                    return
                self._all_gather(p)
            except BaseException as e:
                self.exc = e
            finally:
                self.task_queue.task_done()

    @torch.no_grad()
    def _all_gather(self, p):
        if p.ndim == 0 or p.shape[0] % self.rs_size != 0:
            raise ValueError(f"param shape {tuple(p.shape)} cannot be split by rs_size={self.rs_size}")
        if p.chunk_part.shape[0] != p.shape[0] // self.rs_size:
            raise ValueError("chunk_part does not match rs_size")
        full = p.detach()
        g = C.all_gather_cat(p.chunk_part.detach().contiguous(), self.rs_group)
        full.copy_(g.reshape(full.shape))
        p.state.fill_(1)


def set_opt_hook(model, timeout_s: float = 600.0):
    """Forward pre-hooks: a module runs only once its chunked parameters are
    all-gathered (GPU: the current stream waits for the gather event; CPU: wait
    for the ready byte, bounded by `timeout_s`)."""
    handles = []
    for name, module in model.named_modules():
        own = [p for p in module.parameters(recurse=False) if hasattr(p, "state") and hasattr(p, "chunk_part")]
        if not own:
            continue

        def hook(mod, inputs, own=own):
            for p in own:
                ev = getattr(p, "_harp_ready_event", None)
                if ev is not None:
                    torch.cuda.current_stream(p.device).wait_event(ev)
                    continue
                if p.is_cuda:
                    continue
                t0 = time.time()
                while int(p.state.item()) != 1:
                    if time.time() - t0 > timeout_s:
                        raise TimeoutError(f"parameter of {mod.__class__.__name__} never became ready")
                    time.sleep(1e-5)

        handles.append(module.register_forward_pre_hook(hook))
    return handles
