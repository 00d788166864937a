"""Sequence-parallel autograd functions (reference: managers/shard_manager.py:4-79).

SequenceScatter   forward: keep this rank's chunk of dim 1; backward: all-gather
SequenceAllGather forward: all-gather the chunks along dim 1; backward: own chunk
SPBroadcast       forward: identity; backward: all-reduce (sum) over the SP group

The reference puts a barrier before every collective; stream-ordered NCCL /
harp collectives make that unnecessary.  SPBroadcast's backward sums the
gradient of a replicated input over the SP group: use it only when the
gradients of the parameters that produced the input are NOT summed over SP
ranks again afterwards (the reference's owner-gradient scheme).  Models
trained with harp_b200.trainer.Trainer sum every gradient over all ranks and
therefore do not use it.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..parallel import collectives as C


def _chunk(x: torch.Tensor, group) -> torch.Tensor:
    n, r = C.world(group), C.rank(group)
    return torch.chunk(x, n, dim=1)[r]


def _gather_dim1(x: torch.Tensor, group) -> torch.Tensor:
    n = C.world(group)
    if n == 1:
        return x
    g = C.all_gather_cat(x.contiguous(), group)  # [n, B, s, ...]
    return torch.cat(list(g.unbind(0)), dim=1)


class SequenceScatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, global_unified, sp_group):
        ctx.sp_group = sp_group
        return _chunk(global_unified, sp_group).contiguous()

    @staticmethod
    def backward(ctx, grad_local):
        return _gather_dim1(grad_local, ctx.sp_group), None


class SequenceAllGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local_unified, sp_group):
        ctx.sp_group = sp_group
        return _gather_dim1(local_unified, sp_group)

    @staticmethod
    def backward(ctx, grad_global):
        return _chunk(grad_global, ctx.sp_group).contiguous(), None


class SPBroadcast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input_tensor, sp_group):
        ctx.sp_group = sp_group
        return input_tensor

    @staticmethod
    def backward(ctx, grad_output):
        g = grad_output.contiguous().clone()
        if C.world(ctx.sp_group) > 1:
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=ctx.sp_group)
        return g, None
