"""Fully sharded bf16 weights with the all-gather gated inside the consuming GEMMs.

Reference: managers/weight_manager.py:127-208 (build_chunk_param: each rank owns
row chunks of every weight; AsyncParamAllGatherManager gathers them after the
optimizer step) and the per-op readiness wait of async_rt/runtime.py:66-72 /
cpp_async_runtime.cpp:117-123 (an op spins on `weight.state` before it runs).

Here (TrainConfig(shard_params=True), NVLink communicator, one process per GPU):
  * The 2-D weights of every block (the ModuleList elements) are one gradient
    bucket each; rank r keeps only its 1/world slice of each bucket
    (`ShardedFlatParams.shard`), and the optimizer writes the updated slice back
    there (no push).  Everything else (embedders, final layer, biases, norm
    weights) stays replicated and is pushed by the optimizer as before.
  * Two symmetric staging slots hold whole buckets.  Before block l runs
    (forward, and again before its backward) every rank pushes its slice of
    l's bucket into every rank's slot l % 2 from a side stream (one harp kernel
    of 16-byte peer stores) and release-signals GATH[slot]; a push into a slot
    first waits until every rank has acknowledged all earlier uses of it
    (GACK[slot]).  The next block's gather is issued while the current block
    computes.
  * The block's parameters are re-pointed at their staging slot, and every
    harp GEMM launched for the block carries a device-side gate: each CTA
    waits (bounded) until every rank's GATH[slot] reached the slot's gather
    count before its TMA producer, MMA and epilogue roles start (gemm_sm100.cu
    wait_weight_gate).  Nothing on the host waits for the gather.
  * This rank's own slice is ordered by a stream dependency (the compute
    stream waits for the side stream's push), never by a spin on a flag that
    another kernel of the same GPU sets.
"""
from __future__ import annotations

from functools import partial
from typing import Dict, List, Optional

import torch

from ..trainer import FlatParams


def block_modules(model: torch.nn.Module) -> List[torch.nn.Module]:
    """Elements of the model's top-level ModuleLists, in registration order."""
    mods: List[torch.nn.Module] = []
    for _, child in model.named_children():
        if isinstance(child, torch.nn.ModuleList):
            mods.extend(list(child))
    return mods


def shard_groups(model: torch.nn.Module) -> List[List[torch.Tensor]]:
    """One group per block, last-run block first (backward completion order):
    the block's matrices (parameters with two or more dimensions)."""
    groups = [[p for p in m.parameters() if p.dim() >= 2] for m in block_modules(model)]
    groups = [g for g in groups if g]
    groups.reverse()
    return groups


class ShardedFlatParams(FlatParams):
    """FlatParams whose block buckets are sharded: the flat gradient buffer is
    full size (every rank writes its gradients there and the owners pull-reduce
    them), the replicated parameters (the last bucket) sit at the start of a
    symmetric buffer of their size, and the block buckets' parameters live as
    this rank's slices in `shard`, gathered into staging slots when used."""

    def __init__(self, model: torch.nn.Module, device, comm, align: int = 256):
        self.comm = comm
        super().__init__(model, device, align=align, world=comm.world, buckets=shard_groups(model), rest_first=True)

    def _allocate(self, alloc):
        W = self.comm.world
        rest_hi = self.buckets[self.rest_bucket][1] if self.rest_bucket >= 0 else 0
        self.flat, self.grad = self.comm.allocate_flat(self.numel, param_numel=max(rest_hi, 8 * W))
        self.flat.zero_()
        self.grad.zero_()
        self.shard_off: Dict[int, int] = {}
        tot = 0
        for b, (lo, hi) in enumerate(self.buckets):
            if b != self.rest_bucket:
                self.shard_off[b] = tot
                tot += (hi - lo) // W
        self.shard = torch.zeros(max(tot, 8), device=self.device, dtype=self.dtype)
        sizes = [hi - lo for b, (lo, hi) in enumerate(self.buckets) if b != self.rest_bucket]
        self.slot_numel = max(sizes) if sizes else 8
        self.comm.param_slots(self.slot_numel)
        # block parameters, by bucket: (param, offset within the bucket)
        self.bucket_params: Dict[int, List[tuple]] = {}

    def _place(self):
        W, r = self.comm.world, self.comm.rank
        tmp: Dict[int, torch.Tensor] = {}
        for p, o in zip(self.params, self.offsets):
            b = self.bucket_of[id(p)]
            n = p.numel()
            if b == self.rest_bucket:
                self.flat[o:o + n].copy_(p.data.reshape(-1).to(device=self.device, dtype=self.dtype))
                p.data = self.flat[o:o + n].view(p.shape)
                continue
            lo, hi = self.buckets[b]
            if b not in tmp:
                tmp[b] = torch.zeros(hi - lo, device=self.device, dtype=self.dtype)
            tmp[b][o - lo:o - lo + n].copy_(p.data.reshape(-1).to(device=self.device, dtype=self.dtype))
            self.bucket_params.setdefault(b, []).append((p, o - lo))
        for b, full in tmp.items():
            lo, hi = self.buckets[b]
            nb = (hi - lo) // W
            self.shard[self.shard_off[b]:self.shard_off[b] + nb].copy_(full[r * nb:(r + 1) * nb])
        del tmp
        for b in self.bucket_params:
            self.point(b, 0)  # shape-correct views until the bucket is first gathered

    def point(self, b: int, slot: int):
        """Re-point bucket b's parameters at staging slot `slot`."""
        view = self.comm.slot_view(slot)
        for p, rel in self.bucket_params[b]:
            p.data = view[rel:rel + p.numel()].view(p.shape)

    def local_slice(self, b: int) -> torch.Tensor:
        lo, hi = self.buckets[b]
        nb = (hi - lo) // self.comm.world
        return self.shard[self.shard_off[b]:self.shard_off[b] + nb]

    def segment_param(self, b: int, f: int, n: int) -> torch.Tensor:
        if b == self.rest_bucket:
            return self.flat[f:f + n]
        return self.local_slice(b)

    def local_out(self, b: int) -> Optional[torch.Tensor]:
        return None if b == self.rest_bucket else self.local_slice(b)

    def full_bucket(self, b: int, group) -> torch.Tensor:
        """Bucket b gathered with a torch.distributed collective (cold paths:
        checkpoints, parity checks)."""
        import torch.distributed as dist

        lo, hi = self.buckets[b]
        out = torch.empty(hi - lo, device=self.device, dtype=self.dtype)
        dist.all_gather_into_tensor(out, self.local_slice(b).contiguous(), group=group)
        return out

    def state_dict_views(self, group=None) -> Dict[str, torch.Tensor]:
        full = {b: self.full_bucket(b, group) for b in self.bucket_params}
        out = {}
        for n, p, o in zip(self.names, self.params, self.offsets):
            b = self.bucket_of[id(p)]
            if b == self.rest_bucket:
                out[n] = p.data
            else:
                lo = self.buckets[b][0]
                out[n] = full[b][o - lo:o - lo + p.numel()].view(p.shape)
        return out


class ParamGatherer:
    """Issues the per-block gathers, re-points the block's parameters and sets
    the GEMM gate around the block's forward and backward (module hooks)."""

    def __init__(self, model: torch.nn.Module, flat: ShardedFlatParams, comm, device):
        self.flat, self.comm = flat, comm
        self.stream = torch.cuda.Stream(device=device)
        self.blocks = block_modules(model)
        # bucket of each block (by its first matrix)
        self.block_bucket: List[int] = []
        for m in self.blocks:
            mats = [p for p in m.parameters() if p.dim() >= 2]
            self.block_bucket.append(flat.bucket_of[id(mats[0])] if mats else -1)
        self.bucket_block = {b: l for l, b in enumerate(self.block_bucket) if b >= 0}
        self.step = 0
        self.content: List[Optional[tuple]] = [None, None]
        self._pushed: Dict[int, torch.cuda.Event] = {}
        self._released: set = set()
        self.active = False
        for l, m in enumerate(self.blocks):
            if self.block_bucket[l] >= 0:
                m.register_forward_pre_hook(partial(self._pre_forward, l))
                m.register_forward_hook(partial(self._post_forward, l))

    def begin_step(self):
        self.step += 1
        self.active = True
        self._released = set()

    def end_step(self):
        self.active = False
        self.comm.clear_gate()

    def _ensure(self, l: int):
        b = self.block_bucket[l]
        if b < 0:
            return
        s = l % 2
        if self.content[s] == (b, self.step):
            return
        # behind the compute stream's current point: the acknowledgements of
        # this slot's earlier uses (own included) and the optimizer's writes of
        # the slice are ordered before the push
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        with torch.cuda.stream(self.stream):
            self.comm.gather_slice(s, self.flat.local_slice(b), self.comm.rank * self.flat.local_slice(b).numel())
        done = torch.cuda.Event()
        done.record(self.stream)
        self.content[s] = (b, self.step)
        self._pushed[s] = done

    def _activate(self, l: int):
        s = l % 2
        self._ensure(l)
        # this rank's own slice: a stream dependency, not a flag spin
        torch.cuda.current_stream().wait_event(self._pushed[s])
        self.flat.point(self.block_bucket[l], s)
        self.comm.gate_slot(s)

    def _release(self, l: int):
        s = l % 2
        self.comm.clear_gate()
        self.comm.ack_slot(s)

    def _pre_forward(self, l, module, args):
        if not self.active:
            return None
        self._activate(l)
        if l + 1 < len(self.blocks):
            self._ensure(l + 1)  # prefetch: overlaps this block's compute
        return None

    def _post_forward(self, l, module, args, out):
        if not self.active:
            return None
        self._release(l)
        if isinstance(out, torch.Tensor) and out.requires_grad:
            out.register_hook(partial(self._pre_backward, l))
        return None

    def _pre_backward(self, l, grad):
        if self.active:
            self._activate(l)
            if l - 1 >= 0:
                self._ensure(l - 1)
        return None

    def bucket_done(self, b: int):
        """Bucket b's gradients are complete: its block's backward is over."""
        l = self.bucket_block.get(b)
        if l is not None and self.active and b not in self._released:
            self._released.add(b)
            self._release(l)
