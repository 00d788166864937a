"""Training engine: flat parameter/gradient buffers, ZeRO-1 sharded AdamW,
gradient sync, and the step API used by train.py, bench.py and smoke().

Mapping to the reference:
  * The reference shares one copy of weights and gradients per die through
    POSIX shm, sums SP gradients into it (accumulate_sp/accumulate.cpp), then
    either all-reduces over DP (COMM_MODE 0) or reduce-scatters over the RS
    group, steps AdamW on row chunks and all-gathers the chunks back
    (COMM_MODE 1; managers/weight_manager.py:127-208).
  * Here every rank owns a replica of the bf16 weights in ONE flat buffer
    (parameters are views into it) and a flat bf16 gradient buffer.  After
    backward, gradients are summed over every rank (SP and DP alike) by a
    reduce-scatter of the flat buffer, each rank runs AdamW (fp32 master, m, v)
    on its 1/world shard, and the updated bf16 shards are all-gathered.  That is
    the reference's COMM_MODE 1 with rs_size = world, done on the whole buffer.
  * comm="nvl" routes the reduce-scatter / AdamW / all-gather through the
    NVLink kernels of harp_b200.parallel.nvlink (one fused kernel per bucket).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .models.dit import DiT, flow_matching_loss_local
from .ops import functional as Fn
from .parallel import collectives as C
from .parallel.sequence import SPContext, resolve_mode
from .runtime import errors


@dataclass
class TrainConfig:
    lr: float = 1e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.0
    grad_scale: float = 1.0
    comm: str = "auto"  # "auto" | "torch" | "nvl"
    align: int = 256  # elements; every parameter starts on a 512-byte boundary
    # Capture the whole step (zero-grad, forward, backward, AdamW) in one CUDA
    # graph after `graph_warmup` eager steps and replay it (single-GPU runs).
    cuda_graph: bool = False
    graph_warmup: int = 2


class FlatParams:
    """Packs every parameter of `model` into one contiguous buffer (and one for
    gradients).  Parameters become views; registration order is kept, so
    adjacently registered weights (e.g. SwiGLU w1, w3) stay adjacent."""

    def __init__(self, model: torch.nn.Module, device, dtype=torch.bfloat16, align: int = 256, world: int = 1,
                 alloc=None):
        self.params: List[torch.nn.Parameter] = []
        self.names: List[str] = []
        offs = []
        off = 0
        seen = set()
        prev_end = None
        for name, p in model.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            # keep tightly-packed neighbours contiguous (w1 directly followed by w3)
            if not (name.endswith("w3.weight") and prev_end is not None):
                off = (off + align - 1) // align * align
            offs.append(off)
            self.params.append(p)
            self.names.append(name)
            off += p.numel()
            prev_end = off
        quantum = align * max(1, world)
        self.numel = (off + quantum - 1) // quantum * quantum
        self.offsets = offs
        if alloc is not None:
            # e.g. symmetric (peer-mapped) buffers of the NVLink communicator
            self.flat, self.grad = alloc(self.numel)
            self.flat.zero_()
            self.grad.zero_()
        else:
            self.flat = torch.zeros(self.numel, device=device, dtype=dtype)
            self.grad = torch.zeros(self.numel, device=device, dtype=dtype)
        for p, o in zip(self.params, offs):
            n = p.numel()
            self.flat[o:o + n].copy_(p.data.reshape(-1).to(device=device, dtype=dtype))
            p.data = self.flat[o:o + n].view(p.shape)
        self.attach_grads()

    def attach_grads(self):
        for p, o in zip(self.params, self.offsets):
            p.grad = self.grad[o:o + p.numel()].view(p.shape)
            # fused blocks may store their weight gradients straight into this slot
            p._harp_direct_grad = True

    def zero_grad(self):
        self.grad.zero_()
        # autograd may have replaced a grad view (e.g. after a None grad); re-attach
        for p, o in zip(self.params, self.offsets):
            g = p.grad
            if g is None or g.data_ptr() != self.grad[o:].data_ptr():
                p.grad = self.grad[o:o + p.numel()].view(p.shape)

    def state_dict_views(self) -> Dict[str, torch.Tensor]:
        return {n: p.data for n, p in zip(self.names, self.params)}


class ShardedAdamW:
    """AdamW with fp32 master weights and moments for this rank's 1/world
    slice of the flat parameter buffer."""

    def __init__(self, flat: FlatParams, cfg: TrainConfig, group=None):
        self.flat, self.cfg, self.group = flat, cfg, group
        self.world = C.world(group)
        self.rank = C.rank(group)
        n = flat.numel // self.world
        self.shard_numel = n
        lo = self.rank * n
        self.master = flat.flat[lo:lo + n].float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad_shard = torch.empty(n, device=flat.flat.device, dtype=flat.grad.dtype)
        self.step_count = 0
        self.lr = cfg.lr
        # [lr, 1 - beta1^t, sqrt(1 - beta2^t)] on the device for CUDA-graph replays
        self.hyper: Optional[torch.Tensor] = None
        self._hyper_host: Optional[torch.Tensor] = None

    def use_device_hyper(self):
        """Read lr and the bias corrections from a device tensor that
        `advance()` refreshes before every step (a captured step then replays
        with the current values)."""
        if self.hyper is None:
            self.hyper = torch.zeros(3, device=self.master.device, dtype=torch.float32)
            self._hyper_host = torch.zeros(3, dtype=torch.float32).pin_memory()

    def advance(self):
        """Count the next step and stage its hyper-parameters on the device
        (device-hyper mode; ordered on the current stream)."""
        self.step_count += 1
        t = self.step_count
        self._hyper_host.copy_(torch.tensor([self.lr, 1.0 - self.cfg.beta1 ** t,
                                             math.sqrt(1.0 - self.cfg.beta2 ** t)], dtype=torch.float32))
        self.hyper.copy_(self._hyper_host, non_blocking=True)

    def param_shard(self) -> torch.Tensor:
        n = self.shard_numel
        return self.flat.flat[self.rank * n:(self.rank + 1) * n]

    def step(self, grad_shard: Optional[torch.Tensor] = None):
        if self.hyper is None:
            self.step_count += 1
        g = grad_shard if grad_shard is not None else self.grad_shard
        Fn.adamw_flat(self.master, self.m, self.v, g, self.param_shard(), self.lr, self.cfg.beta1, self.cfg.beta2,
                      self.cfg.eps, self.cfg.weight_decay, max(1, self.step_count), self.cfg.grad_scale,
                      hyper=self.hyper)

    def state_dict(self):
        return {"step": self.step_count, "lr": self.lr, "master": self.master.cpu(), "exp_avg": self.m.cpu(),
                "exp_avg_sq": self.v.cpu(), "rank": self.rank, "world": self.world,
                "shard_numel": self.shard_numel}

    def load_state_dict(self, sd):
        assert sd["world"] == self.world and sd["shard_numel"] == self.shard_numel, "optimizer shard layout mismatch"
        self.step_count = sd["step"]
        self.lr = sd["lr"]
        self.master.copy_(sd["master"])
        self.m.copy_(sd["exp_avg"])
        self.v.copy_(sd["exp_avg_sq"])
        self.param_shard().copy_(self.master.to(self.param_shard().dtype))


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    sp_size: int = 1
    dp_size: int = 1
    world_group: object = None
    sp_group: object = None
    dp_group: object = None
    rs_size: int = 1
    rs_group: object = None

    @staticmethod
    def build(sp_size: Optional[int] = None, rs_size: Optional[int] = None) -> "ParallelState":
        """Groups as the reference's train.py:155-166,234-272: SP groups of
        consecutive ranks (i // sp); DP groups of equal SP index (i % sp); RS
        groups of rs = min(rs_size, world / sp) ranks with equal SP index inside
        blocks of sp * rs ranks (i // (sp * rs) * sp + i % sp)."""
        if not (dist.is_available() and dist.is_initialized()):
            return ParallelState()
        W, r = dist.get_world_size(), dist.get_rank()
        sp = sp_size or W
        assert W % sp == 0, f"world {W} not divisible by sp {sp}"
        dp = W // sp
        rs = max(1, min(rs_size or 1, dp))
        assert dp % rs == 0, f"dp {dp} not divisible by rs {rs}"
        sp_group = dp_group = rs_group = None
        # SP groups: consecutive ranks (the reference's sp_ranks[i // sp]); DP: same local index
        for g in range(dp):
            ranks = list(range(g * sp, (g + 1) * sp))
            pg = dist.new_group(ranks) if sp < W else dist.group.WORLD
            if r in ranks:
                sp_group = pg
        for l in range(sp):
            ranks = list(range(l, W, sp))
            pg = dist.new_group(ranks) if dp > 1 else None
            if r in ranks:
                dp_group = pg
        if rs > 1:
            for blk in range(W // (sp * rs)):
                for l in range(sp):
                    ranks = [blk * sp * rs + j * sp + l for j in range(rs)]
                    pg = dist.new_group(ranks)
                    if r in ranks:
                        rs_group = pg
        return ParallelState(W, r, sp, dp, dist.group.WORLD, sp_group, dp_group, rs, rs_group)


class Trainer:
    """One training step = forward (sequence-parallel), backward, gradient sync,
    sharded AdamW, parameter all-gather.  ``step()`` is the public end-to-end
    call: it takes a (pinned) host batch, copies it to the GPU, trains, and
    returns the loss as a Python float."""

    def __init__(self, model, par: ParallelState, cfg: TrainConfig, device, sp_backend: str = "auto",
                 loss_fn=None, sp_mode: str = "auto"):
        """loss_fn(model, latent, noise, text, sigmas, sp, **extra) -> this rank's share
        of the global loss; defaults to the DiT flow-matching loss."""
        self.model, self.par, self.cfg, self.device = model, par, cfg, device
        self.loss_fn = loss_fn or flow_matching_loss_local
        on_gpu = torch.device(device).type == "cuda"
        self.grad_comm = None
        if par.world_size > 1 and on_gpu and (cfg.comm == "nvl" or (cfg.comm == "auto" and _nvl_available())):
            from .parallel.nvlink import NVLinkComm

            self.grad_comm = NVLinkComm.get(par.world_group, device)
        alloc = self.grad_comm.allocate_flat if self.grad_comm is not None else None
        self.flat = FlatParams(model, device, align=cfg.align, world=par.world_size, alloc=alloc)
        self.opt = ShardedAdamW(self.flat, cfg, par.world_group)
        backend = sp_backend
        comm = None
        if par.sp_size > 1:
            if backend == "auto":
                backend = "nvl" if (on_gpu and _nvl_available()) else "torch"
            if backend == "nvl":
                from .parallel.nvlink import NVLinkComm

                comm = NVLinkComm.get(par.sp_group, device)
        self.sp_comm = comm
        mode = resolve_mode(sp_mode, _model_heads(model), par.sp_size) if par.sp_size > 1 else "ring"
        self.sp = SPContext.from_group(par.sp_group, backend=backend, comm=comm, mode=mode) \
            if par.sp_size > 1 else SPContext()
        self.global_step = 0
        # CUDA-graph state (single GPU): static inputs, the captured step, its loss
        self._graph = None
        self._graph_inputs: Optional[Dict[str, torch.Tensor]] = None
        self._graph_loss: Optional[torch.Tensor] = None
        self._graph_launches = 0
        self._eager_steps = 0
        self.graph_enabled = bool(cfg.cuda_graph) and on_gpu and par.world_size == 1

    # -- device-resident step (inputs already on the GPU) -------------------
    def train_step(self, latent, noise, text, sigmas, **extra) -> torch.Tensor:
        for comm in {id(c): c for c in (self.sp_comm, self.grad_comm) if c is not None}.values():
            comm.begin_step()
        if self.grad_comm is not None:
            # peers' parameter shards of the previous step have landed and they
            # are done reading our gradient buffer: safe to zero it and run
            self.grad_comm.wait_params()
        self.flat.zero_grad()
        loss = self.loss_fn(self.model, latent, noise, text, sigmas, self.sp, **extra)
        if self.par.dp_size > 1:
            loss = loss / self.par.dp_size
        loss.backward()
        self.sync_and_step()
        self.global_step += 1
        lsum = loss.detach().float().reshape(1)
        if self.par.world_size > 1:
            C.all_reduce_sum_(lsum, self.par.world_group)
            # each SP group holds one sample set: undo the dp split and sum of SP partials
        return lsum

    def sync_and_step(self):
        if self.par.world_size == 1:
            self.opt.step(self.flat.grad)
            return
        if self.grad_comm is not None:
            self.grad_comm.rs_adamw_ag(self.flat, self.opt)
            return
        C.reduce_scatter_flat(self.flat.grad, self.opt.grad_shard, self.par.world_group)
        self.opt.step()
        C.all_gather_flat(self.opt.param_shard(), self.flat.flat, self.par.world_group)

    # -- CUDA-graph replay of the whole step (single GPU) ---------------------------
    def run(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        """One step from a batch of device or (pinned) host tensors, returning
        the loss as a device tensor.  With `cuda_graph`, the first
        `graph_warmup` steps run eagerly, the next one is captured, and later
        steps copy the batch into the captured step's inputs and replay it."""
        if self.graph_enabled and not all(isinstance(v, torch.Tensor) for v in batch.values()):
            self.graph_enabled = False  # list-valued inputs (e.g. Z-Image conditions) run eagerly
        if not self.graph_enabled:
            dev = self.device
            b = {k: _to_dev(v, dev) for k, v in batch.items()}
            extra = {k: v for k, v in b.items() if k not in ("latent", "noise", "text", "sigmas")}
            return self.train_step(b["latent"], b["noise"], b["text"], b["sigmas"], **extra)
        if self._graph is None and self._eager_steps < self.cfg.graph_warmup:
            self._eager_steps += 1
            b = {k: _to_dev(v, self.device) for k, v in batch.items()}
            extra = {k: v for k, v in b.items() if k not in ("latent", "noise", "text", "sigmas")}
            return self.train_step(b["latent"], b["noise"], b["text"], b["sigmas"], **extra)
        if self._graph is None:
            try:
                self._capture(batch)
            except RuntimeError as e:  # an op that cannot be captured: stay eager
                import warnings

                warnings.warn(f"harp_b200: CUDA-graph capture of the step failed ({e}); running eagerly")
                self.graph_enabled = False
                self.opt.hyper = None
                return self.run(batch)
        for k, v in batch.items():
            self._graph_inputs[k].copy_(v, non_blocking=True)
        self.opt.advance()
        self._graph.replay()
        torch.ops.harp.add_launch_count(self._graph_launches)
        self.global_step += 1
        return self._graph_loss

    def _capture(self, batch: Dict[str, torch.Tensor]):
        dev = self.device
        self._graph_inputs = {k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in batch.items()}
        for k, v in batch.items():
            self._graph_inputs[k].copy_(v, non_blocking=True)
        self.opt.use_device_hyper()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        b = self._graph_inputs
        extra = {k: v for k, v in b.items() if k not in ("latent", "noise", "text", "sigmas")}
        before = int(torch.ops.harp.launch_count())
        step_count, global_step = self.opt.step_count, self.global_step
        with torch.cuda.graph(graph):
            loss = self.train_step(b["latent"], b["noise"], b["text"], b["sigmas"], **extra)
        # capture recorded the kernels without running them: take back the
        # launch count and step counters it advanced; every replay re-adds them
        self._graph_launches = int(torch.ops.harp.launch_count()) - before
        torch.ops.harp.add_launch_count(-self._graph_launches)
        self.opt.step_count, self.global_step = step_count, global_step
        self._graph, self._graph_loss = graph, loss

    # -- public end-to-end step ------------------------------------------------
    def step(self, batch: Dict[str, torch.Tensor]) -> float:
        """batch: host tensors 'latent' [B,C,H,W], 'noise' [B,C,H,W], 'text' [B,L,Dt], 'sigmas' [B]
        (pinned for asynchronous copies).  Returns the loss (global mean)."""
        if self.graph_enabled:
            return float(self.run(batch).item())
        dev = self.device
        latent = batch["latent"].to(dev, non_blocking=True)
        noise = batch["noise"].to(dev, non_blocking=True)
        text = batch["text"].to(dev, non_blocking=True)
        sigmas = batch["sigmas"].to(dev, non_blocking=True)
        extra = {k: _to_dev(v, dev) for k, v in batch.items() if k not in ("latent", "noise", "text", "sigmas")}
        loss = self.train_step(latent, noise, text, sigmas, **extra)
        return float(loss.item())

    def check_errors(self):
        if torch.device(self.device).type == "cuda":
            errors.check(torch.device(self.device))


def _model_heads(model) -> int:
    cfg = getattr(model, "cfg", None)
    if cfg is not None and hasattr(cfg, "heads"):
        return int(cfg.heads)
    for m in model.modules():
        for attr in ("n_heads", "heads", "num_heads"):
            if isinstance(getattr(m, attr, None), int):
                return int(getattr(m, attr))
    return 1


def _to_dev(v, dev):
    if isinstance(v, torch.Tensor):
        return v.to(dev, non_blocking=True)
    if isinstance(v, (list, tuple)):
        return type(v)(_to_dev(x, dev) for x in v)
    return v


def _nvl_available() -> bool:
    try:
        from .parallel import nvlink  # noqa: F401

        return nvlink.available()
    except Exception:
        return False
