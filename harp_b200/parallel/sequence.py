"""Sequence parallelism: the SP context and the sequence-parallel attention.

Semantics follow the reference's ring attention (gemm/ring_attention/
ring_attn.cpp:2412-2829): the joint sequence is split into `sp` equal chunks,
rank r holds chunk r, and attention for the local queries runs over the keys
and values of every chunk.  The reference reads peers' K/V chunks in place
from die-shared memory in the staggered order (step + rank) % sp; its
backward keeps K/V stationary and reduces the per-rank dQ partials.

Here the forward gathers K/V of all chunks into one key sequence and runs
the tcgen05 flash-attention kernel over it, visiting key tiles from this
rank's own chunk onwards (so compute starts before peers' chunks land when
the NVLink exchange is used).  The backward computes dQ locally and dK/dV
for the whole gathered sequence, then reduce-scatters dK/dV back to the
chunk owners.

Exchange backends:
  "torch"  torch.distributed all-gather / reduce-scatter (gloo or NCCL)
  "nvl"    harp NVLink exchange: peers' K/V pulled over NVLink into a
           local buffer chunk by chunk with per-chunk readiness flags that
           the attention kernel waits on (harp_b200.parallel.nvlink)
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ..ops import functional as Fn
from . import collectives as C


@dataclass
class SPContext:
    size: int = 1
    rank: int = 0
    group: Any = None
    backend: str = "local"  # "local" | "torch" | "nvl"
    comm: Any = None  # harp_b200.parallel.nvlink.NVLinkComm for backend == "nvl"

    @staticmethod
    def single() -> "SPContext":
        return SPContext()

    @staticmethod
    def from_group(group, backend: str = "torch", comm=None) -> "SPContext":
        n = C.world(group)
        if n == 1:
            return SPContext()
        return SPContext(size=n, rank=C.rank(group), group=group, backend=backend, comm=comm)


def _kv_gather_torch(k, v, B, S, HD, sp: SPContext):
    kv_local = torch.cat([k, v], 1)  # [B*S, 2HD]
    g = C.all_gather_cat(kv_local, sp.group)  # [sp, B*S, 2HD]
    return g.view(sp.size, B, S, 2 * HD).permute(1, 0, 2, 3).reshape(B * sp.size * S, 2 * HD).contiguous()


def _dkv_scatter_torch(dkv_full, B, S, HD, sp: SPContext):
    per_rank = dkv_full.view(B, sp.size, S, 2 * HD).permute(1, 0, 2, 3).contiguous()  # [sp, B, S, 2HD]
    return C.reduce_scatter_sum(per_rank.view(sp.size, B * S, 2 * HD), sp.group)


def sp_attention_forward(q, k, v, B: int, S: int, H: int, Dh: int, sp: SPContext):
    """q, k, v: local [B*S, >=H*Dh] token-major.  Returns (o [B*S, H*Dh], saved)."""
    HD = H * Dh
    if sp.size == 1:
        o, lse = Fn.attn_fwd(q, k, v, B, S, S, H, Dh)
        return o, {"lse": lse}
    if sp.backend == "nvl" and sp.comm is not None:
        kv_full, ready, epoch = sp.comm.kv_exchange(k, v, B, S, HD)
        start_tile = (sp.rank * S) // 128
        o, lse = Fn.attn_fwd(q, kv_full[:, :HD], kv_full[:, HD:], B, S, sp.size * S, H, Dh, ready=ready,
                             chunk_len=S, start_tile=start_tile, epoch=epoch)
        return o, {"lse": lse, "kv": kv_full}
    kv_full = _kv_gather_torch(k, v, B, S, HD, sp)
    o, lse = Fn.attn_fwd(q, kv_full[:, :HD], kv_full[:, HD:], B, S, sp.size * S, H, Dh)
    return o, {"lse": lse, "kv": kv_full}


def sp_attention_backward(saved, q, k, v, o, do, B: int, S: int, H: int, Dh: int, sp: SPContext,
                          dv_out: Optional[torch.Tensor] = None):
    """Returns (dq, dk) for the local chunk; dV is written into `dv_out` (or returned
    as a third value when dv_out is None)."""
    HD = H * Dh
    lse = saved["lse"]
    if sp.size == 1:
        dq, dk, dv = Fn.attn_bwd(q, k, v, o, do, lse, B, S, S, H, Dh, dv_out=dv_out)
        return (dq, dk) if dv_out is not None else (dq, dk, dv)
    kv_full = saved["kv"]
    Skv = sp.size * S
    if sp.backend == "nvl" and sp.comm is not None:
        dkv_full = sp.comm.dkv_buffer(B * Skv, 2 * HD, q.dtype)
    else:
        dkv_full = torch.empty(B * Skv, 2 * HD, device=q.device, dtype=q.dtype)
    dq, _, _ = Fn.attn_bwd(q, kv_full[:, :HD], kv_full[:, HD:], o, do, lse, B, S, Skv, H, Dh,
                           dk_out=dkv_full[:, :HD], dv_out=dkv_full[:, HD:])
    if sp.backend == "nvl" and sp.comm is not None:
        dkv = sp.comm.dkv_reduce_scatter(dkv_full, B, S, HD)
    else:
        dkv = _dkv_scatter_torch(dkv_full, B, S, HD, sp)
    dk = dkv[:, :HD]
    if dv_out is not None:
        dv_out.copy_(dkv[:, HD:])
        return dq, dk
    return dq, dk, dkv[:, HD:]
