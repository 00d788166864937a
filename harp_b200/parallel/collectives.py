"""Backend-neutral collective helpers over torch.distributed process groups.

The NVLink fused paths (harp_b200.parallel.nvlink) replace these on the hot
path; these serve the gloo (CPU) tests, the NCCL fallback and cold paths.
"""
from __future__ import annotations


import torch
import torch.distributed as dist


def world(group=None) -> int:
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def rank(group=None) -> int:
    if not dist.is_available() or not dist.is_initialized():
        return 0
    return dist.get_rank(group)


def _is_gloo(group) -> bool:
    try:
        return dist.get_backend(group) == "gloo"
    except Exception:
        return False


def all_gather_cat(x: torch.Tensor, group=None) -> torch.Tensor:
    """Stack of every rank's `x` along a new leading dim, in group-rank order."""
    n = world(group)
    if n == 1:
        return x.unsqueeze(0)
    x = x.contiguous()
    out = torch.empty((n,) + tuple(x.shape), device=x.device, dtype=x.dtype)
    if _is_gloo(group):
        dist.all_gather(list(out.unbind(0)), x, group=group)
    else:
        dist.all_gather_into_tensor(out, x, group=group)
    return out


def all_to_all(x: torch.Tensor, group=None) -> torch.Tensor:
    """x: [n, ...] (slab j goes to rank j) -> [n, ...] with slab j = what rank j sent here."""
    n = world(group)
    if n == 1:
        return x.clone()
    x = x.contiguous()
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=group)
    return out


def reduce_scatter_sum(x: torch.Tensor, group=None) -> torch.Tensor:
    """x: [n, ...] (one slab per rank) -> sum over ranks of slab[my rank]."""
    n = world(group)
    if n == 1:
        return x[0]
    x = x.contiguous()
    if _is_gloo(group):
        y = x.clone()
        dist.all_reduce(y, group=group)
        return y[rank(group)].contiguous()
    out = torch.empty(tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
    dist.reduce_scatter_tensor(out, x, group=group)
    return out


def all_reduce_sum_(x: torch.Tensor, group=None) -> torch.Tensor:
    if world(group) > 1:
        dist.all_reduce(x, group=group)
    return x


def reduce_scatter_flat(flat: torch.Tensor, shard: torch.Tensor, group=None) -> torch.Tensor:
    """Sum `flat` (length n*len(shard)) over ranks and keep this rank's slice."""
    n = world(group)
    if n == 1:
        shard.copy_(flat)
        return shard
    if _is_gloo(group):
        y = flat.clone()
        dist.all_reduce(y, group=group)
        r = rank(group)
        shard.copy_(y[r * shard.numel():(r + 1) * shard.numel()])
        return shard
    dist.reduce_scatter_tensor(shard, flat, group=group)
    return shard


def all_gather_flat(shard: torch.Tensor, flat: torch.Tensor, group=None) -> torch.Tensor:
    n = world(group)
    if n == 1:
        if flat.data_ptr() != shard.data_ptr():
            flat.copy_(shard)
        return flat
    if _is_gloo(group):
        parts = list(flat.view(n, -1).unbind(0))
        dist.all_gather(parts, shard.contiguous(), group=group)
        return flat
    dist.all_gather_into_tensor(flat, shard.contiguous(), group=group)
    return flat
