"""Training engine: flat parameter/gradient buffers, ZeRO-1 sharded AdamW,
gradient sync, and the step API used by train.py, bench.py and smoke().

Mapping to the reference:
  * The reference shares one copy of weights and gradients per die through
    POSIX shm, sums SP gradients into it (accumulate_sp/accumulate.cpp), then
    either all-reduces over DP (COMM_MODE 0) or reduce-scatters over the RS
    group, steps AdamW on row chunks and all-gathers the chunks back
    (COMM_MODE 1; managers/weight_manager.py:127-208).
  * Here every rank owns a replica of the bf16 weights in ONE flat buffer
    (parameters are views into it) and a flat bf16 gradient buffer, laid out
    bucket by bucket: a bucket is a group of consecutive blocks (in the order
    their backward finishes) and every rank owns an equal 1/world slice of
    every bucket.  Gradients are summed over every rank (SP and DP alike) by a
    reduce-scatter of each bucket, each rank runs AdamW (fp32 master, m, v) on
    its slices, and the updated bf16 slices are all-gathered.  That is the
    reference's COMM_MODE 1 with rs_size = world.
  * comm="nvl": the moment a bucket's last gradient is written (the fused
    blocks report their direct gradient writes, autograd reports the rest
    through post-accumulate hooks), the rank signals its peers on the compute
    stream and enqueues ONE fused kernel for that bucket on a side stream:
    pull-reduce of its slice from every peer over NVLink, AdamW, and a push of
    the new bf16 slice into every peer's parameter buffer
    (harp_b200.parallel.nvlink).  These kernels run while the backward of the
    earlier blocks continues, as the reference's grad-ready hooks feed its
    communication threads (managers/grad_manager.py:41-159,
    accumulate_sp/accumulate.cpp:389-484).  Buckets are enqueued in one fixed
    order on every rank.
"""
from __future__ import annotations

import contextlib
import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .models.dit import flow_matching_loss_local
from .ops import functional as Fn
from .parallel import collectives as C
from .parallel.sequence import SPContext, resolve_mode
from .runtime import errors
from .utils.observability import phase


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
    # graph after `graph_warmup` eager steps and replay it (1 GPU, or N GPUs
    # whose exchanges all run on the NVLink communicator).
    cuda_graph: bool = False
    graph_warmup: int = 2
    # multi-GPU NVLink gradient sync: send each bucket (about this many
    # parameters) as soon as its gradients are complete, overlapping the rest
    # of the backward; False = one fused kernel over everything after backward
    overlap_grad_sync: bool = True
    bucket_params: int = 64_000_000
    # multi-GPU NVLink: keep only this rank's 1/world slice of every block's
    # weights and gather a block's weights into a staging slot right before it
    # runs, gated inside its GEMMs (harp_b200.parallel.param_shard)
    shard_params: bool = False
    # keep the fp32 master weights and AdamW moments in pinned, mapped host
    # memory (the optimizer kernels read and write them over the host link)
    offload_optimizer: bool = False
    # move activations saved for backward to pinned host memory during the
    # forward and back during the backward (managers.mem_manager.HBMToDDROffloader)
    offload_activations: bool = False


class FlatParams:
    """Packs every parameter of `model` into one contiguous buffer (and one for
    gradients).  Parameters become views; registration order is kept inside a
    bucket, so adjacently registered weights (e.g. SwiGLU w1, w3) stay adjacent.

    `buckets` (optional) is a list of parameter groups; the flat layout holds
    them one after the other, each starting on a world*align boundary and
    padded to a multiple of it, so that every rank owns an equal, aligned
    1/world slice of every bucket.  Parameters in no group form a last bucket.
    ``self.buckets`` lists each bucket's [lo, hi) range of the flat buffer."""

    def __init__(self, model: torch.nn.Module, device, dtype=torch.bfloat16, align: int = 256, world: int = 1,
                 alloc=None, buckets: Optional[List[List[torch.Tensor]]] = None, rest_first: bool = False):
        self._layout(model, align, world, buckets, rest_first)
        self.device, self.dtype = device, dtype
        self._allocate(alloc)
        self._place()
        self.attach_grads()

    def _layout(self, model, align, world, buckets, rest_first):
        """Offsets of every parameter: bucket by bucket (the last bucket holds
        the parameters no group names; with rest_first it goes first in
        memory but keeps the last index)."""
        self.params: List[torch.nn.Parameter] = []
        self.names: List[str] = []
        named = []
        seen = set()
        for name, p in model.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            named.append((name, p))
        order = {id(p): i for i, (_, p) in enumerate(named)}
        groups: List[List[int]] = []
        placed = set()
        for grp in buckets or []:
            idx = sorted({order[id(p)] for p in grp if id(p) in order and id(p) not in placed})
            placed.update(id(named[i][1]) for i in idx)
            if idx:
                groups.append(idx)
        rest = [i for i, (_, p) in enumerate(named) if id(p) not in placed]
        self.rest_bucket = len(groups) if rest else -1
        if rest:
            groups.append(rest)
        mem_order = list(range(len(groups)))
        if rest_first and rest:
            mem_order = [len(groups) - 1] + mem_order[:-1]
        quantum = align * max(1, world)
        offs = []
        off = 0
        self.buckets: List[tuple] = [(0, 0)] * len(groups)
        self.bucket_of: Dict[int, int] = {}
        for gi in mem_order:
            idx = groups[gi]
            off = (off + quantum - 1) // quantum * quantum
            lo = off
            prev_end = None
            for i in idx:
                name, p = named[i]
                # keep tightly-packed neighbours contiguous (w1 directly followed by w3)
                if not (name.endswith("w3.weight") and prev_end is not None):
                    off = (off + align - 1) // align * align
                offs.append(off)
                self.params.append(p)
                self.names.append(name)
                self.bucket_of[id(p)] = gi
                off += p.numel()
                prev_end = off
            off = (off + quantum - 1) // quantum * quantum
            self.buckets[gi] = (lo, off)
        self.numel = max(off, quantum)
        if not self.buckets:
            self.buckets.append((0, self.numel))
        self.offsets = offs

    def _allocate(self, alloc):
        if alloc is not None:
            # e.g. symmetric (peer-mapped) buffers of the NVLink communicator
            self.flat, self.grad = alloc(self.numel)
            self.flat.zero_()
            self.grad.zero_()
        else:
            self.flat = torch.zeros(self.numel, device=self.device, dtype=self.dtype)
            self.grad = torch.zeros(self.numel, device=self.device, dtype=self.dtype)

    def _place(self):
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.flat[o:o + n].copy_(p.data.reshape(-1).to(device=self.device, dtype=self.dtype))
            p.data = self.flat[o:o + n].view(p.shape)

    # hooks for the sharded-parameter variant (harp_b200.parallel.param_shard)
    def segment_param(self, b: int, f: int, n: int) -> torch.Tensor:
        """This rank's bf16 slice [f, f + n) of bucket b."""
        return self.flat[f:f + n]

    def local_out(self, b: int) -> Optional[torch.Tensor]:
        """Where the optimizer writes bucket b's new slice when it is not
        pushed to every rank (None: pushed)."""
        return None

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
    slice of every bucket of the flat parameter buffer.  The slices are
    concatenated in bucket order into one state vector; ``segments`` lists
    (flat offset, length, state offset) per bucket."""

    def __init__(self, flat: FlatParams, cfg: TrainConfig, group=None):
        self.flat, self.cfg, self.group = flat, cfg, group
        self.world = C.world(group)
        self.rank = C.rank(group)
        self.segments: List[tuple] = []
        off = 0
        for lo, hi in flat.buckets:
            n = (hi - lo) // self.world
            self.segments.append((lo + self.rank * n, n, off))
            off += n
        self.shard_numel = off
        dev = flat.grad.device
        ctx = contextlib.nullcontext()
        if cfg.offload_optimizer and dev.type == "cuda":
            from .runtime import alloc

            ctx = alloc.use_tier("host", dev.index)  # pinned, mapped host memory
        with ctx:
            self.master = torch.cat([flat.segment_param(b, f, n).float()
                                     for b, (f, n, _) in enumerate(self.segments)])
            self.m = torch.zeros_like(self.master)
            self.v = torch.zeros_like(self.master)
        self.grad_shard = torch.empty(off, device=flat.flat.device, dtype=flat.grad.dtype)
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

    def param_segments(self) -> List[torch.Tensor]:
        """bf16 views of the parameter slices that this rank's state covers."""
        return [self.flat.segment_param(b, f, n) for b, (f, n, _) in enumerate(self.segments)]

    def local_param_out(self, b: int) -> Optional[torch.Tensor]:
        """Destination of bucket b's updated slice when it stays with this rank
        (sharded parameters); None when the update is pushed to every rank."""
        return self.flat.local_out(b)

    def grad_segments(self, grad: torch.Tensor) -> List[torch.Tensor]:
        return [grad[f:f + n] for f, n, _ in self.segments]

    def step(self, grad_shard: Optional[torch.Tensor] = None):
        """AdamW on this rank's slices.  grad_shard: the summed gradient in state
        order (default: self.grad_shard); with one rank the flat gradient buffer
        itself may be passed."""
        if self.hyper is None:
            self.step_count += 1
        g = grad_shard if grad_shard is not None else self.grad_shard
        for (f, n, o), p in zip(self.segments, self.param_segments()):
            gs = g[f:f + n] if (self.world == 1 and g.numel() == self.flat.numel) else g[o:o + n]
            Fn.adamw_flat(self.master[o:o + n], self.m[o:o + n], self.v[o:o + n], gs, p, self.lr, self.cfg.beta1,
                          self.cfg.beta2, self.cfg.eps, self.cfg.weight_decay, max(1, self.step_count),
                          self.cfg.grad_scale, hyper=self.hyper)

    def state_dict(self):
        return {"step": self.step_count, "lr": self.lr, "master": self.master.cpu(), "exp_avg": self.m.cpu(),
                "exp_avg_sq": self.v.cpu(), "rank": self.rank, "world": self.world,
                "shard_numel": self.shard_numel, "segments": [list(s) for s in self.segments]}

    def load_state_dict(self, sd):
        assert sd["world"] == self.world and sd["shard_numel"] == self.shard_numel, "optimizer shard layout mismatch"
        if "segments" in sd:
            assert [tuple(s) for s in sd["segments"]] == self.segments, "optimizer shard layout mismatch"
        self.step_count = sd["step"]
        self.lr = sd["lr"]
        self.master.copy_(sd["master"])
        self.m.copy_(sd["exp_avg"])
        self.v.copy_(sd["exp_avg_sq"])
        for (f, n, o), p in zip(self.segments, self.param_segments()):
            p.copy_(self.master[o:o + n].to(p.dtype))


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
        self.gatherer = None
        if cfg.shard_params and par.world_size > 1:
            if self.grad_comm is None:
                raise ValueError("shard_params needs the NVLink communicator (comm='nvl' on GPUs)")
            from .parallel.param_shard import ParamGatherer, ShardedFlatParams

            self.flat = ShardedFlatParams(model, device, self.grad_comm, align=cfg.align)
            self.gatherer = ParamGatherer(model, self.flat, self.grad_comm, device)
        else:
            buckets = grad_buckets(model, cfg.bucket_params) if par.world_size > 1 else None
            self.flat = FlatParams(model, device, align=cfg.align, world=par.world_size, alloc=alloc,
                                   buckets=buckets)
        self.opt = ShardedAdamW(self.flat, cfg, par.world_group)
        # overlapped gradient sync: buckets go out as their gradients complete
        # (sharded parameters always overlap: a block's staging slot is released
        # when its gradients are reported)
        self._overlap = self.grad_comm is not None and (cfg.overlap_grad_sync or self.gatherer is not None) and \
            len(self.flat.buckets) > 1
        self._ready: set = set()
        self._next_bucket = 0
        self._bucket_left: List[int] = []
        self._sync_active = False
        self._comm_stream = None
        if self._overlap:
            self._comm_stream = torch.cuda.Stream(device=device)
            for p in self.flat.params:
                p.register_post_accumulate_grad_hook(self._on_grad_ready)
                p._harp_grad_ready = self._on_grad_ready
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
        # CUDA-graph state: static inputs, the captured step, its loss
        self._graph = None
        self._graph_inputs: Optional[Dict[str, torch.Tensor]] = None
        self._graph_loss: Optional[torch.Tensor] = None
        self._graph_launches = 0
        self._eager_steps = 0
        self._replays = 0
        self._epoch_incr: Dict[int, Dict[str, int]] = {}
        # multi-GPU steps are captured when every exchange is an NVLink kernel
        # (their flag values then come from the device: NVLinkComm.begin_capture)
        multi_ok = (self.grad_comm is not None and (par.sp_size == 1 or self.sp_comm is not None)
                    and os.environ.get("HARP_GRAPH_MULTI", "1") != "0")
        self.graph_enabled = bool(cfg.cuda_graph) and on_gpu and (par.world_size == 1 or multi_ok)

    # -- device-resident step (inputs already on the GPU) -------------------
    def _comms(self):
        return list({id(c): c for c in (self.sp_comm, self.grad_comm) if c is not None}.values())

    def train_step(self, latent, noise, text, sigmas, **extra) -> torch.Tensor:
        epochs0 = {id(c): dict(c.epoch) for c in self._comms()}
        for comm in self._comms():
            comm.begin_step()
        if self.grad_comm is not None:
            # peers' parameter shards of the previous step have landed and they
            # are done reading our gradient buffer: safe to zero it and run
            self.grad_comm.wait_params()
        self.flat.zero_grad()
        self._begin_sync()
        if self.gatherer is not None:
            self.gatherer.begin_step()
        with phase("forward"), self._saved_tensor_ctx():
            loss = self.loss_fn(self.model, latent, noise, text, sigmas, self.sp, **extra)
            if self.par.dp_size > 1:
                loss = loss / self.par.dp_size
        with phase("backward"):
            loss.backward()
        with phase("grad_sync_optimizer"):
            self.sync_and_step()
        if self.gatherer is not None:
            self.gatherer.end_step()
        self.global_step += 1
        lsum = loss.detach().float().reshape(1)
        if self.par.world_size > 1:
            C.all_reduce_sum_(lsum, self.par.world_group)
            # each SP group holds one sample set: undo the dp split and sum of SP partials
        # increments of every flag counter over one step (what a captured step
        # adds per replay)
        self._epoch_incr = {id(c): {k: v - epochs0[id(c)].get(k, 0) for k, v in c.epoch.items()}
                            for c in self._comms()}
        return lsum

    def _saved_tensor_ctx(self):
        if not self.cfg.offload_activations or torch.device(self.device).type != "cuda":
            return contextlib.nullcontext()
        if getattr(self, "_offloader", None) is None:
            from .managers.mem_manager import HBMToDDROffloader

            self._offloader = HBMToDDROffloader()
        return torch.autograd.graph.saved_tensors_hooks(self._offloader.pack_hook, self._offloader.unpack_hook)

    # -- gradient sync -----------------------------------------------------------
    def _begin_sync(self):
        """Start of a step's backward: count the step, reset the bucket marks."""
        if not self._overlap:
            return
        self.grad_comm.begin_grad_sync(self.opt)
        self._ready = set()
        self._next_bucket = 0
        self._bucket_left = [0] * len(self.flat.buckets)
        for p in self.flat.params:
            self._bucket_left[self.flat.bucket_of[id(p)]] += 1
        self._sync_active = True

    def _on_grad_ready(self, p):
        """A parameter's gradient of this step is complete (enqueued on the
        current stream): mark it and send every bucket that is complete, in
        bucket order."""
        if not self._sync_active or id(p) in self._ready:
            return
        self._ready.add(id(p))
        b = self.flat.bucket_of[id(p)]
        self._bucket_left[b] -= 1
        if self._bucket_left[b] == 0 and self.gatherer is not None:
            self.gatherer.bucket_done(b)
        self._launch_ready()

    def _launch_ready(self, flush: bool = False):
        nb = len(self.flat.buckets)
        while self._next_bucket < nb and (flush or self._bucket_left[self._next_bucket] == 0):
            self.grad_comm.rs_adamw_bucket(self.flat, self.opt, self._next_bucket, self._comm_stream)
            self._next_bucket += 1

    def sync_and_step(self):
        if self.par.world_size == 1:
            self.opt.step(self.flat.grad)
            return
        if self.grad_comm is not None:
            if self._overlap:
                if self.gatherer is not None:  # blocks whose gradients nothing reported
                    for b, left in enumerate(self._bucket_left):
                        if left > 0:
                            self.gatherer.bucket_done(b)
                self._launch_ready(flush=True)  # buckets whose gradients nothing reported
                self._sync_active = False
                self.grad_comm.end_grad_sync(self._comm_stream)
            else:
                self.grad_comm.rs_adamw_ag(self.flat, self.opt)
            return
        g = self.opt.grad_shard
        for (lo, hi), (f, n, o) in zip(self.flat.buckets, self.opt.segments):
            C.reduce_scatter_flat(self.flat.grad[lo:hi], g[o:o + n], self.par.world_group)
        self.opt.step()
        for (lo, hi), p in zip(self.flat.buckets, self.opt.param_segments()):
            C.all_gather_flat(p, self.flat.flat[lo:hi], self.par.world_group)

    # -- CUDA-graph replay of the whole step ----------------------------------------
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
                if self.par.world_size > 1:
                    raise  # every rank must take the same path
                import warnings

                warnings.warn(f"harp_b200: CUDA-graph capture of the step failed ({e}); running eagerly")
                self.graph_enabled = False
                self.opt.hyper = None
                return self.run(batch)
        for k, v in batch.items():
            self._graph_inputs[k].copy_(v, non_blocking=True)
        self.opt.advance()
        if self._replays > 0:  # the captured flag values are those of the first replay
            for c in self._comms():
                c.step_delta.add_(1)
        self._replays += 1
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
        comms = self._comms()
        for c in comms:  # flag values of the captured kernels advance per replay on the device
            c.begin_capture(self._epoch_incr.get(id(c), {}))
        try:
            with torch.cuda.graph(graph):
                loss = self.train_step(b["latent"], b["noise"], b["text"], b["sigmas"], **extra)
        finally:
            for c in comms:
                c.end_capture()
        self._replays = 0
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

    def model_state_dict(self) -> Dict[str, torch.Tensor]:
        """The model's state dict with every parameter's current value (with
        sharded parameters a collective: every rank must call it)."""
        sd = self.model.state_dict()
        if self.gatherer is not None:
            views = self.flat.state_dict_views(self.par.world_group)
            sd.update({k: v for k, v in views.items() if k in sd})
        return sd

    def close(self):
        """Release the captured step (it may hold NCCL work: release it before
        the process group goes away)."""
        self._graph = None
        self._graph_loss = None
        self._graph_inputs = None

    def check_errors(self):
        if torch.device(self.device).type == "cuda":
            errors.check(torch.device(self.device))


def grad_buckets(model: torch.nn.Module, target: int) -> List[List[torch.Tensor]]:
    """Parameter groups in the order their gradients complete in backward:
    the elements of the model's top-level ModuleLists (blocks), last-run
    first, merged into groups of about `target` parameters.  Parameters
    outside those lists (embedders, final layer) are left to the last group
    that FlatParams forms from whatever no group holds."""
    units: List[List[torch.Tensor]] = []
    for _, child in model.named_children():
        if isinstance(child, torch.nn.ModuleList):
            units.extend([list(m.parameters()) for m in child])
    units.reverse()  # lists registered (and run) later finish their backward first
    groups: List[List[torch.Tensor]] = []
    cur: List[torch.Tensor] = []
    size = 0
    for u in units:
        cur.extend(u)
        size += sum(p.numel() for p in u)
        if size >= target:
            groups.append(cur)
            cur, size = [], 0
    if cur:
        groups.append(cur)
    return groups


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
