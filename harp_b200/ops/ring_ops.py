"""The reference's ring-attention operator names on harp kernels.

    torch.ops.ring_attention_ops.ring_attention_forward(q, k, v, out, m_i, l_i, sp_size, scale)
    torch.ops.ring_attention_ops.ring_attention_backward(q, grad_q, k, dK, v, dV, grad_out, m_i, l_i, D,
                                                        sp_size, scale)

Same schemas and tensor contract as gemm/ring_attention/
torch_ring_attention_ops.cpp:260-268 (q, k, v [B, H, T_local, D] bf16
token-major views; out fp32 [B, H, T, D]; running max m_i bf16 and sum l_i
fp32 [B, H, T, 1]; D = rowsum(dO * O) fp32), so code written against the
reference's op library runs unchanged.  Here the statistics encode the
log-sum-exp: m_i = bf16(lse) and l_i = exp(lse - m_i), i.e.
lse = m_i + log(l_i) exactly as the reference combines them, and the
backward takes the LSE and D from its arguments.  The ops gather the K/V
chunks of the SP group set with set_sp_context() (sp_size must match its
size) and run the harp attention kernels with any softmax scale; on CPU
tensors they use the fp32 restatements.  `CPURingAttention` is the
reference's autograd wrapper (src/models/z_image/module/attn.py:15-50).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import functional as Fn
from ..parallel.sequence import SPContext, _dkv_scatter_torch, _kv_gather_torch

_ctx: SPContext = SPContext()
_lib = torch.library.Library("ring_attention_ops", "DEF")
_lib.define("ring_attention_forward(Tensor q, Tensor k, Tensor v, Tensor(a!) out, Tensor(b!) m_i, Tensor(c!) l_i, "
            "int sp_size, float scale) -> (Tensor(a!), Tensor(b!), Tensor(c!))")
_lib.define("ring_attention_backward(Tensor q, Tensor(a!) grad_q, Tensor k, Tensor(b!) dK, Tensor v, Tensor(c!) dV, "
            "Tensor grad_out, Tensor m_i, Tensor l_i, Tensor D, int sp_size, float scale) "
            "-> (Tensor(a!), Tensor(b!), Tensor(c!))")


def set_sp_context(sp: Optional[SPContext]) -> None:
    """SP group the ring_attention_ops run over (default: a single rank)."""
    global _ctx
    _ctx = sp or SPContext()


def _tok(x: torch.Tensor) -> torch.Tensor:
    """[B, H, T, D] view of token-major storage -> [B*T, H*D]."""
    B, H, T, D = x.shape
    return x.transpose(1, 2).reshape(B * T, H * D)


def _check(sp_size: int):
    if sp_size != _ctx.size:
        raise RuntimeError(f"ring_attention_ops: sp_size {sp_size} but the SP context has {_ctx.size} ranks "
                           "(harp_b200.ops.ring_ops.set_sp_context)")


def _gather_kv(kt, vt, B, T, HD):
    """Every rank's K|V chunk of the SP group, sample-major [B*sp*T, 2*HD]
    (the reference's ring passes the same chunks around its dies)."""
    if _ctx.size == 1:
        return torch.cat([kt, vt], 1)
    return _kv_gather_torch(kt, vt, B, T, HD, _ctx)


def _forward(q, k, v, out, m_i, l_i, sp_size, scale):
    """Attention of the local queries over the keys of every SP rank, with the
    given softmax scale."""
    _check(sp_size)
    B, H, T, D = q.shape
    HD = H * D
    qt = _tok(q).contiguous()
    kv = _gather_kv(_tok(k).contiguous(), _tok(v).contiguous(), B, T, HD)
    o, lse = Fn.attn_fwd(qt, kv[:, :HD], kv[:, HD:], B, T, _ctx.size * T, H, D, scale=scale)
    lse = lse.view(B, H, -1)[:, :, :T]
    out.copy_(o.view(B, T, H, D).transpose(1, 2))
    m_i.copy_(lse.unsqueeze(-1))
    l_i.copy_(torch.exp(lse.unsqueeze(-1) - m_i.float()))
    return out, m_i, l_i


def _backward(q, grad_q, k, dK, v, dV, grad_out, m_i, l_i, D, sp_size, scale):
    """Uses the forward's statistics as the op contract passes them: the
    log-sum-exp is m_i + log(l_i) and D = rowsum(dO * O) is the softmax
    backward's row term, so nothing of the forward is recomputed; only the K/V
    chunks are gathered again (they are not part of the contract), and the
    dK/dV of every chunk are summed back to its owner."""
    _check(sp_size)
    B, H, T, Dh = q.shape
    HD = H * Dh
    W = _ctx.size
    qt, kt, vt = _tok(q).contiguous(), _tok(k).contiguous(), _tok(v).contiguous()
    ld = Fn.lse_ld(T)
    lse = torch.full((B, H, ld), float("inf"), device=q.device, dtype=torch.float32)
    lse[:, :, :T] = (m_i.float() + torch.log(l_i.float()))[..., 0]
    delta = torch.zeros((B, H, ld), device=q.device, dtype=torch.float32)
    delta[:, :, :T] = D.float()[..., 0]
    kv = _gather_kv(kt, vt, B, T, HD)
    dq, dk, dv = Fn.attn_bwd(qt, kv[:, :HD], kv[:, HD:], None, _tok(grad_out).contiguous(), lse.reshape(-1), B, T,
                             W * T, H, Dh, scale=scale, delta=delta.reshape(-1))
    if W > 1:
        dkv = _dkv_scatter_torch(torch.cat([dk, dv], 1), B, T, HD, _ctx)
        dk, dv = dkv[:, :HD], dkv[:, HD:]
    grad_q.copy_(dq.view(B, T, H, Dh).transpose(1, 2))
    dK.copy_(dk.reshape(B, T, H, Dh).transpose(1, 2))
    dV.copy_(dv.reshape(B, T, H, Dh).transpose(1, 2))
    return grad_q, dK, dV


for _key in ("CPU", "CUDA"):
    _lib.impl("ring_attention_forward", _forward, _key)
    _lib.impl("ring_attention_backward", _backward, _key)


class CPURingAttention(torch.autograd.Function):
    """Reference autograd wrapper around the two ops (name kept for API parity;
    it runs on whatever device its inputs live on)."""

    @staticmethod
    def forward(ctx, local_q, local_k, local_v, sp_size):
        scale = 1.0 / math.sqrt(local_q.size(-1))
        out = torch.zeros_like(local_q, dtype=torch.float32)
        shape = local_q.shape[:3] + (1,)
        m_i = torch.full(shape, float("-inf"), device=local_q.device, dtype=torch.bfloat16)
        l_i = torch.empty(shape, device=local_q.device, dtype=torch.float32)
        torch.ops.ring_attention_ops.ring_attention_forward(local_q, local_k, local_v, out, m_i, l_i, sp_size, scale)
        ctx.save_for_backward(local_q, local_k, local_v, out, m_i, l_i)
        ctx.sp_size, ctx.scale = sp_size, scale
        return out.to(local_q.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, m_i, l_i = ctx.saved_tensors
        D = torch.sum(grad_out.float() * out, dim=-1, keepdim=True)
        gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        torch.ops.ring_attention_ops.ring_attention_backward(q, gq, k, gk, v, gv, grad_out.contiguous(), m_i, l_i, D,
                                                             ctx.sp_size, ctx.scale)
        return gq, gk, gv, None
