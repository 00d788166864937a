"""Gradient synchronisation overlapped with backward (reference:
managers/grad_manager.py:1-186 driving accumulate_sp/accumulate.cpp).

Per parameter, in the deterministic order its post-accumulate-grad hook fires:
  1. SP sum: parameters whose forward ran on the rank's own sequence chunk get
     their gradient summed over the SP group.  Parameters computed on
     replicated inputs already hold the full gradient on every SP rank and only
     the owner's copy is kept - the reference encodes this with
     expected_count 4 / 1, hard-wired to sp=4 and to the Z-Image parameter
     names (grad_manager.py:53-61); here `replicated(name)` decides and the SP
     size comes from the group.
  2. The owner copies the result into `p.shared_grad` and runs the data-parallel
     communication chosen by COMM_MODE (accumulate.cpp:419-465):
       0  all-reduce over the DP group
       1  reduce-scatter rows over the RS group into p.chunk_part.grad, then
          all-reduce that chunk over the DP group
       2  all-reduce over the RS group, then all-reduce the chunk over DP
  3. p.grad is released.
On CUDA the work for each parameter is enqueued on a side stream as soon as its
hook fires (after an event recorded on the producing stream), so it overlaps
the rest of backward; on CPU (gloo) it runs in hook order at
wait_for_completion().
"""
from __future__ import annotations

import os
import time
from typing import Callable, Dict, List, Optional, Set

import torch
import torch.distributed as dist

from ..parallel import collectives as C
from .weight_manager import is_norm_param


def reference_replicated(name: str) -> bool:
    """The reference's rule: only transformer blocks run on sequence chunks."""
    return not any(k in name for k in ("layers.", "context_refiner.", "noise_refiner.", "cond_refiner_"))


class AsyncGradSyncManager:
    def __init__(self, model, local_rank: int, local_die: int, param_rank: Dict[int, int], my_params_set: Set,
                 sp_group=None, dp_group=None, rs_group=None, comm_mode: Optional[int] = None,
                 replicated: Callable[[str], bool] = reference_replicated):
        self.local_rank, self.local_die = local_rank, local_die
        self.param_rank, self.my_params_set = param_rank, my_params_set
        self.sp_group, self.dp_group, self.rs_group = sp_group, dp_group, rs_group
        self.comm_mode = int(os.environ.get("COMM_MODE", "0")) if comm_mode is None else comm_mode
        self.disable_dp = os.environ.get("DISABLE_DP", "0") == "1"
        self.replicated = replicated
        self._pending: List = []
        self._stream = None
        self._times = {"tq": 0.0, "sp": 0.0, "dp": 0.0}
        self._hooks = []
        self._worker_exc: Optional[BaseException] = None
        for name, p in reversed(list(model.named_parameters())):
            if p.requires_grad:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._make_hook(name)))

    def _owner(self, name, p) -> bool:
        return is_norm_param(name) or self.param_rank.get(id(p), self.local_rank) == self.local_rank

    def _make_hook(self, name: str):
        def hook(p):
            if p.grad is None:
                return
            if p.grad.is_cuda:
                if self._stream is None:
                    self._stream = torch.cuda.Stream(device=p.grad.device)
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(p.grad.device))
                self._stream.wait_event(ev)
                with torch.cuda.stream(self._stream):
                    try:
                        self._sync(name, p)
                    except BaseException as e:
                        self._worker_exc = e
            else:
                self._pending.append((name, p))

        return hook

    @torch.no_grad()
    def _sync(self, name: str, p):
        g = p.grad
        t0 = time.time()
        if not self.replicated(name) and C.world(self.sp_group) > 1:
            dist.all_reduce(g, group=self.sp_group)
        self._times["sp"] += time.time() - t0
        t0 = time.time()
        if self._owner(name, p):
            dst = getattr(p, "shared_grad", None)
            if dst is None:
                dst = g
            elif dst.data_ptr() != g.data_ptr():
                dst.copy_(g)
            if not self.disable_dp:
                self._dp_comm(p, dst)
        self._times["dp"] += time.time() - t0
        p.grad = None

    def _dp_comm(self, p, full):
        chunk = getattr(p, "chunk_part", None)
        if self.comm_mode == 0 or chunk is None:
            C.all_reduce_sum_(full, self.dp_group)
            return
        if self.comm_mode == 1:
            part = torch.empty_like(chunk.grad) if chunk.grad is not None else torch.empty_like(chunk)
            C.reduce_scatter_flat(full.reshape(-1), part.reshape(-1), self.rs_group)
        else:
            C.all_reduce_sum_(full, self.rs_group)
            part = full[chunk.chunk_begin:chunk.chunk_end].clone()
        C.all_reduce_sum_(part, self.dp_group)
        if chunk.grad is None:
            chunk.grad = part
        elif chunk.grad.data_ptr() != part.data_ptr():
            chunk.grad.copy_(part)

    def wait_for_completion(self):
        t0 = time.time()
        pending, self._pending = self._pending, []
        for name, p in pending:
            self._sync(name, p)
        tq = time.time() - t0
        if self._stream is not None:
            torch.cuda.current_stream(self._stream.device).wait_stream(self._stream)
        if self._worker_exc is not None:
            raise RuntimeError("gradient synchronisation failed") from self._worker_exc
        t0 = time.time()
        if dist.is_initialized():
            dist.barrier()
        barr = time.time() - t0
        sp, dp = self._times["sp"], self._times["dp"]
        self._times = {"tq": 0.0, "sp": 0.0, "dp": 0.0}
        return tq, sp, dp, barr

    def shutdown(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
