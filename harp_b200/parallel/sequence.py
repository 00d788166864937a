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

Ulysses mode (mode="ulysses", heads divisible by sp): instead of gathering
K/V, an all-to-all turns the sequence-sharded q, k, v into head-sharded ones
over the FULL sequence (rank r keeps heads [r*H/sp, (r+1)*H/sp)), attention
runs locally, and a second all-to-all returns the output to sequence
sharding.  Per rank and layer this moves 4 x (local activation) x (sp-1)/sp
bytes each way instead of 2 x sp x (local K/V) for the gather, i.e. about
sp/2 times less traffic at sp >= 4.  The reference has no Ulysses mode.

Exchange backends:
  "torch"  torch.distributed all-gather / reduce-scatter (gloo or NCCL)
  "nvl"    harp NVLink exchange (harp_b200.parallel.nvlink): ring mode's
           QK-norm/RoPE kernel stores K/V into every rank's gathered buffer,
           the attention kernel waits per key tile for the flag of the chunk
           it reads, and the attention backward stores each chunk's dK/dV
           into its owner's receive buffer; Ulysses mode's exchanges are
           fused with their producers the same way
"""
from __future__ import annotations

from dataclasses import dataclass
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
    mode: str = "ring"  # "ring" (gather K/V) | "ulysses" (head all-to-all)

    @staticmethod
    def single() -> "SPContext":
        return SPContext()

    @staticmethod
    def from_group(group, backend: str = "torch", comm=None, mode: str = "ring") -> "SPContext":
        n = C.world(group)
        if n == 1:
            return SPContext()
        return SPContext(size=n, rank=C.rank(group), group=group, backend=backend, comm=comm, mode=mode)


def resolve_mode(mode: str, heads: int, sp_size: int) -> str:
    """"auto": Ulysses when the heads split evenly over the SP ranks (it moves
    2x fewer bytes than the K/V gather at sp=4 and 4x fewer at sp=8, and its
    fused NVLink form measured faster from sp=2 on), else the K/V gather."""
    if mode == "auto":
        return "ulysses" if sp_size > 1 and heads % sp_size == 0 else "ring"
    if mode == "ulysses" and heads % sp_size != 0:
        raise ValueError(f"ulysses SP needs heads ({heads}) divisible by sp ({sp_size})")
    return mode


def _seq_to_heads(ts, B, S, H, Dh, sp: SPContext) -> torch.Tensor:
    """Sequence-sharded [B*S, >=H*Dh] tensors -> head-sharded [T, B*sp*S, (H/sp)*Dh]
    over the full sequence (global token order: chunk-major)."""
    N, Hn = sp.size, H // sp.size
    x = torch.stack([t[:, :H * Dh].reshape(B, S, N, Hn, Dh) for t in ts], 0)  # [T, B, S, N, Hn, Dh]
    recv = C.all_to_all(x.permute(3, 0, 1, 2, 4, 5).contiguous(), sp.group)  # [N(chunk), T, B, S, Hn, Dh]
    return recv.permute(1, 2, 0, 3, 4, 5).reshape(len(ts), B * N * S, Hn * Dh)


def _heads_to_seq(ts, B, S, H, Dh, sp: SPContext) -> torch.Tensor:
    """Head-sharded [B*sp*S, (H/sp)*Dh] tensors -> sequence-sharded [T, B*S, H*Dh]."""
    N, Hn = sp.size, H // sp.size
    x = torch.stack([t.reshape(B, N, S, Hn, Dh) for t in ts], 0)  # [T, B, N(chunk), S, Hn, Dh]
    recv = C.all_to_all(x.permute(2, 0, 1, 3, 4, 5).contiguous(), sp.group)  # [N(head grp), T, B, S, Hn, Dh]
    return recv.permute(1, 2, 3, 0, 4, 5).reshape(len(ts), B * S, H * Dh)


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
    if sp.mode == "ulysses":
        Hn, Sf = H // sp.size, sp.size * S
        qkv_f = _seq_to_heads((q, k, v), B, S, H, Dh, sp)
        o_f, lse = Fn.attn_fwd(qkv_f[0], qkv_f[1], qkv_f[2], B, Sf, Sf, Hn, Dh)
        o = _heads_to_seq((o_f,), B, S, H, Dh, sp)[0]
        return o, {"lse": lse, "qkv_f": qkv_f, "o_f": o_f}
    if ring_nvl(sp):
        o, _, _, _, saved = sp.comm.ring_forward(q, k, v, B, S, H, Dh, q_ready=True)
        return o, saved
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
    if sp.mode == "ulysses":
        Hn, Sf = H // sp.size, sp.size * S
        qkv_f, o_f = saved["qkv_f"], saved["o_f"]
        do_f = _seq_to_heads((do,), B, S, H, Dh, sp)[0]
        dq_f, dk_f, dv_f = Fn.attn_bwd(qkv_f[0], qkv_f[1], qkv_f[2], o_f, do_f, lse, B, Sf, Sf, Hn, Dh)
        dqkv = _heads_to_seq((dq_f, dk_f, dv_f), B, S, H, Dh, sp)
        if dv_out is not None:
            dv_out.copy_(dqkv[2])
            return dqkv[0], dqkv[1]
        return dqkv[0], dqkv[1], dqkv[2]
    kv_full = saved["kv"]
    Skv = sp.size * S
    if ring_nvl(sp):
        dq, dkv = sp.comm.ring_backward(saved, q, o, do, B, S, H, Dh)
    else:
        dkv_full = torch.empty(B * Skv, 2 * HD, device=q.device, dtype=q.dtype)
        dq, _, _ = Fn.attn_bwd(q, kv_full[:, :HD], kv_full[:, HD:], o, do, lse, B, S, Skv, H, Dh,
                               dk_out=dkv_full[:, :HD], dv_out=dkv_full[:, HD:])
        dkv = _dkv_scatter_torch(dkv_full, B, S, HD, sp)
    dk = dkv[:, :HD]
    if dv_out is not None:
        dv_out.copy_(dkv[:, HD:])
        return dq, dk
    return dq, dk, dkv[:, HD:]


def ring_nvl(sp: SPContext) -> bool:
    """The fused NVLink ring path (K/V stored into every rank by their
    producer, attention consuming chunks as their flags arrive, dK/dV stored
    into their owners by the attention backward)."""
    return sp.size > 1 and sp.mode == "ring" and sp.backend == "nvl" and sp.comm is not None


def ulysses_nvl(sp: SPContext) -> bool:
    """The fused NVLink Ulysses path (head all-to-all inside harp kernels)."""
    return sp.size > 1 and sp.mode == "ulysses" and sp.backend == "nvl" and sp.comm is not None


def qkv_attention_forward(qkv, B: int, S: int, H: int, Dh: int, wq, wk, freqs, eps: float, do_norm: bool,
                          sp: SPContext):
    """QK-norm + RoPE of the pre-norm q|k|v rows, then sequence-parallel
    attention.  Returns (o [B*S, H*Dh], rstd_q, rstd_k, q, k, saved); q and k
    (post-norm, this rank's rows) are None on the fused Ulysses path, whose
    exchange applies the norm on the way."""
    HD = H * Dh
    if ulysses_nvl(sp):
        o, rq, rk, saved = sp.comm.uly_forward(qkv, B, S, H, Dh, wq, wk, freqs, eps, do_norm)
        return o, rq, rk, None, None, saved
    if ring_nvl(sp):
        o, q, rq, rk, saved = sp.comm.ring_forward(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], B, S, H, Dh,
                                                   wq, wk, freqs, eps, do_norm)
        return o, rq, rk, q, None, saved
    q, k, rq, rk = Fn.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, eps, do_norm=do_norm)
    o, saved = sp_attention_forward(q, k, qkv[:, 2 * HD:], B, S, H, Dh, sp)
    return o, rq, rk, q, k, saved


def qkv_attention_backward(saved, qkv, q, k, o, do, rq, rk, wq, wk, freqs, do_norm: bool, B: int, S: int, H: int,
                           Dh: int, sp: SPContext, dqkv: Optional[torch.Tensor] = None):
    """Backward of qkv_attention_forward: returns (d qkv_pre [B*S, 3*H*Dh],
    dwq, dwk) (norm-weight gradients fp32, or None)."""
    HD = H * Dh
    if ulysses_nvl(sp):
        g = sp.comm.uly_backward(saved, do, B, S, H, Dh)
        # d(post-RoPE q, k) -> d(pre-norm q, k) in place (one warp per row and head
        # reads its gradient before writing the result); dv is already final
        dwq, dwk = Fn.qknorm_rope_bwd(g[:, :HD], g[:, HD:2 * HD], qkv, rq, rk, H, Dh, wq, wk, freqs, do_norm, g,
                                      want_dw=do_norm)
        return g, dwq, dwk
    if dqkv is None:
        dqkv = torch.empty(B * S, 3 * HD, device=qkv.device, dtype=qkv.dtype)
    if ring_nvl(sp):
        # dK|dV land summed in dqkv[:, HD:3HD]; d(post-RoPE k) -> d(pre-norm k) in place
        dq, _ = sp.comm.ring_backward(saved, q, o, do, B, S, H, Dh, out=dqkv[:, HD:], out_ld=3 * HD)
        dwq, dwk = Fn.qknorm_rope_bwd(dq, dqkv[:, HD:2 * HD], qkv, rq, rk, H, Dh, wq, wk, freqs, do_norm, dqkv,
                                      want_dw=do_norm)
        return dqkv, dwq, dwk
    dq, dk = sp_attention_backward(saved, q, k, qkv[:, 2 * HD:], o, do, B, S, H, Dh, sp, dv_out=dqkv[:, 2 * HD:])
    dwq, dwk = Fn.qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, do_norm, dqkv, want_dw=do_norm)
    return dqkv, dwq, dwk
