"""Functional wrappers over the sm_100a kernels, with CPU restatements.

Every op here has exactly two paths:
  * CUDA tensors -> the harp_b200 CUDA library (``torch.ops.harp.*``).  The
    library is required there: if it is missing, :func:`_native.require`
    raises instead of silently running PyTorch ops.
  * CPU tensors  -> a plain PyTorch fp32 restatement of the same math, used by
    the gloo multi-process tests and as the numerical oracle of the kernels.

Conventions: activations are token-major 2-D views ``[rows, cols]`` (rows =
batch * local sequence); per-sample modulation vectors are ``[B, cols]`` and a
row r belongs to sample ``r // rows_per_batch``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import _native
from ..runtime import errors

EPI_STORE = 0
EPI_STORE_F32 = 1
EPI_ACCUM = 2
EPI_ACCUM_F32 = 3
EPI_GATED_RESIDUAL = 4
EPI_GATED_RESIDUAL_SAVE = 5


def _cuda(t: torch.Tensor) -> bool:
    if t.is_cuda:
        _native.require()
        return True
    return False


def _bcast(v: torch.Tensor, rows_per_batch: int) -> torch.Tensor:
    return v.repeat_interleave(rows_per_batch, 0)


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    out: Optional[torch.Tensor] = None,
    bias: Optional[torch.Tensor] = None,
    epi: int = EPI_STORE,
    alpha: float = 1.0,
    residual: Optional[torch.Tensor] = None,
    gate: Optional[torch.Tensor] = None,
    rows_per_batch: int = 0,
    out2: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """C = alpha * op(a) @ op(b) (+ bias) with an epilogue.

    ``a`` is [M, K] (or [K, M] when ``a_mn``); ``b`` is [N, K] (or [K, N] when
    ``b_mn``) - i.e. the default computes ``a @ b.T`` like ``F.linear``.
    """
    M = a.shape[1] if a_mn else a.shape[0]
    K = a.shape[0] if a_mn else a.shape[1]
    N = b.shape[1] if b_mn else b.shape[0]
    f32 = epi in (EPI_STORE_F32, EPI_ACCUM_F32)
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=torch.float32 if f32 else torch.bfloat16)
    if _cuda(a):
        torch.ops.harp.gemm(a, a_mn, b, b_mn, out, M, N, K, bias, epi, alpha, residual, gate,
                            rows_per_batch, errors.word(a.device), False, out2)
        return out
    am = a.float().t() if a_mn else a.float()
    bm = b.float() if b_mn else b.float().t()
    acc = alpha * (am @ bm)
    if bias is not None:
        acc = acc + bias.float()
    if epi == EPI_GATED_RESIDUAL_SAVE:
        out2.copy_(acc.to(out2.dtype))
        acc = out2.float()
    if epi in (EPI_GATED_RESIDUAL, EPI_GATED_RESIDUAL_SAVE):
        acc = residual.float() + _bcast(gate.float(), rows_per_batch or M) * acc
    elif epi in (EPI_ACCUM, EPI_ACCUM_F32):
        acc = acc + out.float()
    out.copy_(acc.to(out.dtype))
    return out


def linear_fwd(x2d: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    return gemm(x2d, w, bias=b)


def linear_bwd(dy: torch.Tensor, x2d: torch.Tensor, w: torch.Tensor, need_bias: bool,
               dw_out: Optional[torch.Tensor] = None, accumulate: bool = False):
    """dX = dY W ; dW = dY^T X ; db = sum_rows dY."""
    dx = gemm(dy, w, b_mn=True)
    if dw_out is not None:
        gemm(dy, x2d, a_mn=True, b_mn=True, out=dw_out,
             epi=(EPI_ACCUM_F32 if dw_out.dtype == torch.float32 else EPI_ACCUM) if accumulate
             else (EPI_STORE_F32 if dw_out.dtype == torch.float32 else EPI_STORE))
        dw = dw_out
    else:
        dw = gemm(dy, x2d, a_mn=True, b_mn=True)
    db = colsum(dy) if need_bias else None
    return dx, dw, db


# ---------------------------------------------------------------------------
# reductions
# ---------------------------------------------------------------------------
def rows_per_block(rows_per_batch: int) -> int:
    for r in (32, 16, 8, 4, 2, 1):
        if rows_per_batch % r == 0:
            return r
    return 1


def reduce_partials(part: torch.Tensor, per_group: int, groups: int, out_dtype=torch.float32,
                    out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    D = part.shape[1]
    if out is None:
        out = torch.empty(groups, D, device=part.device, dtype=out_dtype)
    if _cuda(part):
        torch.ops.harp.reduce_partials(part, per_group, out, accumulate)
        return out
    s = part.view(groups, -1, D).sum(1) if per_group * groups == part.shape[0] else torch.stack(
        [part[g * per_group:(g + 1) * per_group].sum(0) for g in range(groups)])
    if accumulate:
        s = s + out.float()
    out.copy_(s.to(out.dtype))
    return out


def colsum(x: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Column sums of a [R, D] bf16 matrix (bias gradients)."""
    R, D = x.shape
    if _cuda(x):
        rpb = 64
        part = torch.empty((R + rpb - 1) // rpb, D, device=x.device, dtype=torch.float32)
        torch.ops.harp.colsum_partial(x, rpb, part)
        return reduce_partials(part, part.shape[0], 1, out_dtype).view(D)
    return x.float().sum(0).to(out_dtype)


# ---------------------------------------------------------------------------
# RMSNorm (+ adaLN modulation)
# ---------------------------------------------------------------------------
def rmsnorm_mod_fwd(x: torch.Tensor, w: Optional[torch.Tensor], scale: Optional[torch.Tensor],
                    shift: Optional[torch.Tensor], rows_per_batch: int, eps: float,
                    out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    R, D = x.shape
    y = out if out is not None else torch.empty_like(x)
    rstd = torch.empty(R, device=x.device, dtype=torch.float32)
    if _cuda(x):
        torch.ops.harp.rmsnorm_mod_fwd(x, w, scale, shift, rows_per_batch, eps, y, rstd, False)
        return y, rstd
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    v = xf * r[:, None]
    if w is not None:
        v = v * w.float()
    if scale is not None:
        v = v * (1 + _bcast(scale.float(), rows_per_batch))
    if shift is not None:
        v = v + _bcast(shift.float(), rows_per_batch)
    y.copy_(v.to(y.dtype))
    rstd.copy_(r)
    return y, rstd


def rmsnorm_mod_bwd(x, rstd, dy, w, scale, rows_per_batch, dres=None, want_dw=False, want_mod=False):
    """Returns (dx, dw [D] fp32 or None, dscale [B,D] fp32 or None, dshift [B,D] fp32 or None)."""
    R, D = x.shape
    B = R // rows_per_batch
    if _cuda(x):
        rpb = rows_per_block(rows_per_batch)
        nblk = R // rpb
        pw = torch.empty(nblk, D, device=x.device) if want_dw and w is not None else None
        ps = torch.empty(nblk, D, device=x.device) if want_mod and scale is not None else None
        pb = torch.empty(nblk, D, device=x.device) if want_mod else None
        dx = torch.empty_like(x)
        torch.ops.harp.rmsnorm_mod_bwd(x, rstd, dy, w, scale, rows_per_batch, dres, dx, pw, ps, pb, rpb)
        dw = reduce_partials(pw, nblk, 1).view(D) if pw is not None else None
        ds = reduce_partials(ps, rows_per_batch // rpb, B) if ps is not None else None
        dsh = reduce_partials(pb, rows_per_batch // rpb, B) if pb is not None else None
        return dx, dw, ds, dsh
    xf, g = x.float(), dy.float()
    xh = xf * rstd[:, None]
    s1 = 1 + _bcast(scale.float(), rows_per_batch) if scale is not None else 1.0
    ww = w.float() if w is not None else 1.0
    gs = g * s1
    dxh = gs * ww
    mu = (dxh * xh).mean(-1, keepdim=True)
    dx = rstd[:, None] * (dxh - xh * mu)
    if dres is not None:
        dx = dx + dres.float()
    dw = (gs * xh).sum(0) if (want_dw and w is not None) else None
    ds = (g * xh * ww).view(B, rows_per_batch, D).sum(1) if (want_mod and scale is not None) else None
    dsh = g.view(B, rows_per_batch, D).sum(1) if want_mod else None
    return dx.to(x.dtype), dw, ds, dsh


def layernorm_mod_fwd(x, scale, shift, rows_per_batch, eps):
    R, D = x.shape
    y = torch.empty_like(x)
    mean = torch.empty(R, device=x.device)
    rstd = torch.empty(R, device=x.device)
    if _cuda(x):
        torch.ops.harp.layernorm_mod_fwd(x, scale, shift, rows_per_batch, eps, y, mean, rstd)
        return y, mean, rstd
    xf = x.float()
    mu = xf.mean(-1)
    var = xf.var(-1, unbiased=False)
    r = torch.rsqrt(var + eps)
    v = (xf - mu[:, None]) * r[:, None]
    if scale is not None:
        v = v * (1 + _bcast(scale.float(), rows_per_batch))
    if shift is not None:
        v = v + _bcast(shift.float(), rows_per_batch)
    y.copy_(v.to(y.dtype))
    mean.copy_(mu)
    rstd.copy_(r)
    return y, mean, rstd


def layernorm_mod_bwd(x, mean, rstd, dy, scale, rows_per_batch, want_mod=True):
    R, D = x.shape
    B = R // rows_per_batch
    if _cuda(x):
        rpb = rows_per_block(rows_per_batch)
        nblk = R // rpb
        ps = torch.empty(nblk, D, device=x.device) if (want_mod and scale is not None) else None
        pb = torch.empty(nblk, D, device=x.device) if want_mod else None
        dx = torch.empty_like(x)
        torch.ops.harp.layernorm_mod_bwd(x, mean, rstd, dy, scale, rows_per_batch, dx, ps, pb, rpb)
        ds = reduce_partials(ps, rows_per_batch // rpb, B) if ps is not None else None
        dsh = reduce_partials(pb, rows_per_batch // rpb, B) if pb is not None else None
        return dx, ds, dsh
    xf, g = x.float(), dy.float()
    xh = (xf - mean[:, None]) * rstd[:, None]
    s1 = 1 + _bcast(scale.float(), rows_per_batch) if scale is not None else 1.0
    gs = g * s1
    dx = rstd[:, None] * (gs - gs.mean(-1, keepdim=True) - xh * (gs * xh).mean(-1, keepdim=True))
    ds = (g * xh).view(B, rows_per_batch, D).sum(1) if (want_mod and scale is not None) else None
    dsh = g.view(B, rows_per_batch, D).sum(1) if want_mod else None
    return dx.to(x.dtype), ds, dsh


# ---------------------------------------------------------------------------
# QK-norm + RoPE
# ---------------------------------------------------------------------------
def _rope_cpu(x, cos, sin, inverse=False):
    x0, x1 = x[..., 0::2], x[..., 1::2]
    if inverse:
        o0 = x0 * cos + x1 * sin
        o1 = -x0 * sin + x1 * cos
    else:
        o0 = x0 * cos - x1 * sin
        o1 = x0 * sin + x1 * cos
    return torch.stack([o0, o1], -1).flatten(-2)


def qknorm_rope_fwd(qkv: torch.Tensor, H: int, Dh: int, wq, wk, freqs: Optional[torch.Tensor], eps: float,
                    do_norm: bool = True):
    """qkv [R, >=2*H*Dh] (q at col 0, k at H*Dh).  freqs: fp32 [F, Dh/2, 2] (cos, sin);
    row r uses freqs[r % F].  Returns q_out, k_out [R, H*Dh], rstd_q, rstd_k [R*H]."""
    R = qkv.shape[0]
    qo = torch.empty(R, H * Dh, device=qkv.device, dtype=qkv.dtype)
    ko = torch.empty_like(qo)
    rq = torch.empty(R * H, device=qkv.device) if do_norm else None
    rk = torch.empty(R * H, device=qkv.device) if do_norm else None
    frows = freqs.shape[0] if freqs is not None else 1
    if _cuda(qkv):
        torch.ops.harp.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, frows, eps, do_norm, qo, ko, rq, rk)
        return qo, ko, rq, rk

    def one(x, w, r_out):
        xr = x.float().view(R, H, Dh)
        if do_norm:
            r = torch.rsqrt(xr.pow(2).mean(-1) + eps)
            r_out.copy_(r.view(-1))
            xr = xr * r[..., None]
            if w is not None:
                xr = xr * w.float()
        if freqs is not None:
            idx = torch.arange(R) % frows
            f = freqs[idx]
            xr = _rope_cpu(xr, f[:, None, :, 0], f[:, None, :, 1])
        return xr.reshape(R, H * Dh).to(qkv.dtype)

    qo.copy_(one(qkv[:, : H * Dh], wq, rq))
    ko.copy_(one(qkv[:, H * Dh: 2 * H * Dh], wk, rk))
    return qo, ko, rq, rk


_SMS = {}


def _num_sms(device) -> int:
    idx = torch.device(device).index or 0
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, do_norm, dqkv, want_dw=True):
    """Writes d(q_pre), d(k_pre) into dqkv[:, :2*H*Dh]; returns (dwq, dwk) fp32 or None."""
    R = qkv.shape[0]
    frows = freqs.shape[0] if freqs is not None else 1
    if _cuda(qkv):
        # about 4 blocks per SM; a block's 32 item slots (4 threads per head)
        # each stride over ~ipb/32 (row, head) items
        ipb = max(128, -(-R * H // (4 * _num_sms(qkv.device))))
        nblk = (R * H + ipb - 1) // ipb
        want = want_dw and do_norm and wq is not None
        pwq = torch.empty(nblk, Dh, device=qkv.device) if want else None
        pwk = torch.empty(nblk, Dh, device=qkv.device) if want else None
        torch.ops.harp.qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, frows, do_norm, dqkv, pwq, pwk, ipb)
        if want:
            return reduce_partials(pwq, nblk, 1).view(Dh), reduce_partials(pwk, nblk, 1).view(Dh)
        return None, None

    def one(g, x, w, r):
        gr = g.float().view(R, H, Dh)
        if freqs is not None:
            idx = torch.arange(R) % frows
            f = freqs[idx]
            gr = _rope_cpu(gr, f[:, None, :, 0], f[:, None, :, 1], inverse=True)
        if not do_norm:
            return gr.reshape(R, H * Dh), None
        xr = x.float().view(R, H, Dh)
        rr = r.view(R, H, 1)
        xh = xr * rr
        ww = w.float() if w is not None else 1.0
        dxh = gr * ww
        mu = (dxh * xh).mean(-1, keepdim=True)
        dx = rr * (dxh - xh * mu)
        dw = (gr * xh).sum((0, 1)) if w is not None else None
        return dx.reshape(R, H * Dh), dw

    dxq, dwq = one(dq, qkv[:, : H * Dh], wq, rq)
    dxk, dwk = one(dk, qkv[:, H * Dh: 2 * H * Dh], wk, rk)
    dqkv[:, : H * Dh].copy_(dxq.to(dqkv.dtype))
    dqkv[:, H * Dh: 2 * H * Dh].copy_(dxk.to(dqkv.dtype))
    return (dwq, dwk) if want_dw else (None, None)


# ---------------------------------------------------------------------------
# SwiGLU, gated residual backward
# ---------------------------------------------------------------------------
def swiglu_fwd(gu: torch.Tensor, F_: int) -> torch.Tensor:
    h = torch.empty(gu.shape[0], F_, device=gu.device, dtype=gu.dtype)
    if _cuda(gu):
        torch.ops.harp.swiglu_fwd(gu, h)
        return h
    g, u = gu[:, :F_].float(), gu[:, F_: 2 * F_].float()
    h.copy_((torch.nn.functional.silu(g) * u).to(h.dtype))
    return h


def swiglu_bwd(dh: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    F_ = dh.shape[1]
    dgu = torch.empty(gu.shape[0], 2 * F_, device=gu.device, dtype=gu.dtype)
    if _cuda(gu):
        torch.ops.harp.swiglu_bwd(dh, gu, dgu)
        return dgu
    g, u, d = gu[:, :F_].float(), gu[:, F_: 2 * F_].float(), dh.float()
    s = torch.sigmoid(g)
    dgu[:, :F_].copy_((d * u * s * (1 + g * (1 - s))).to(dgu.dtype))
    dgu[:, F_:].copy_((d * g * s).to(dgu.dtype))
    return dgu


def gate_bwd(dy, a, gate, rows_per_batch, want_bias=True):
    """out = res + gate[b]*a :  returns da = dy*gate, dgate [B, D] fp32, dbias [D] fp32."""
    R, D = dy.shape
    B = R // rows_per_batch
    if _cuda(dy):
        rpb = rows_per_block(rows_per_batch)
        nblk = R // rpb
        da = torch.empty_like(dy)
        pg = torch.empty(nblk, D, device=dy.device)
        pb = torch.empty(nblk, D, device=dy.device) if want_bias else None
        torch.ops.harp.gate_bwd(dy, a, gate, rows_per_batch, da, pg, pb, rpb)
        dgate = reduce_partials(pg, rows_per_batch // rpb, B)
        dbias = reduce_partials(pb, nblk, 1).view(D) if want_bias else None
        return da, dgate, dbias
    g = _bcast(gate.float(), rows_per_batch)
    da = dy.float() * g
    dgate = (dy.float() * a.float()).view(B, rows_per_batch, D).sum(1)
    dbias = da.sum(0) if want_bias else None
    return da.to(dy.dtype), dgate, dbias


def lse_ld(S: int) -> int:
    """Row stride of the per-(batch, head) LSE / delta buffers: S rounded up to a key tile."""
    return (S + 127) // 128 * 128


def rowdot(a: torch.Tensor, b: torch.Tensor, H: int, Dh: int, S: int) -> torch.Tensor:
    """delta[b, h, s] = sum_d a[b*S+s, h, d] * b[b*S+s, h, d]; layout [B, H, lse_ld(S)] (0 past S)."""
    R = a.shape[0]
    B = R // S
    ld = lse_ld(S)
    out = torch.zeros(B * H * ld, device=a.device)
    if _cuda(a):
        torch.ops.harp.rowdot(a, b, H, Dh, S, out)
        return out
    d = (a.float().view(B, S, H, Dh) * b.float().view(B, S, H, Dh)).sum(-1).permute(0, 2, 1)
    out.view(B, H, ld)[:, :, :S].copy_(d)
    return out


def silu(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    if _cuda(x) and x.dtype == torch.bfloat16 and x.is_contiguous():
        torch.ops.harp.elementwise(0, x, None, 0.0, out)
        return out
    return torch.nn.functional.silu(x.float()).to(x.dtype)


def silu_bwd(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    if _cuda(x) and x.dtype == dy.dtype == torch.bfloat16 and x.is_contiguous() and dy.is_contiguous():
        torch.ops.harp.elementwise(1, dy, x, 0.0, out)
        return out
    s = torch.sigmoid(x.float())
    return (dy.float() * s * (1 + x.float() * (1 - s))).to(x.dtype)


# ---------------------------------------------------------------------------
# attention (local; ring variants live in harp_b200.parallel.ring_attention)
# ---------------------------------------------------------------------------
def attn_fwd(q, k, v, B, Sq, Skv, H, Dh, scale=None, ready=None, chunk_len=0, start_tile=0, epoch=0,
             timeout_s=10.0, out=None, q_rot=0, wait_q=False, step_delta=None, epoch_per_step=0):
    """q [B*Sq, >=H*Dh], k/v [B*Skv, >=H*Dh] token-major.  Returns (o [B*Sq, H*Dh],
    lse fp32 [B, H, lse_ld(Sq)] natural log, +inf past Sq).  With `ready`, key
    (and, with wait_q, query) rows of chunk c = row // chunk_len are used only
    once ready[c] >= epoch; q_rot rotates the order of the 256-query pairs."""
    scale = scale if scale is not None else 1.0 / math.sqrt(Dh)
    o = out if out is not None else torch.empty(B * Sq, H * Dh, device=q.device, dtype=q.dtype)
    lse = torch.full((B * H * lse_ld(Sq),), float("inf"), device=q.device)
    if _cuda(q):
        torch.ops.harp.attn_fwd(q, k, v, B, Sq, Skv, H, Dh, scale, o, lse, ready, chunk_len, start_tile, epoch,
                                timeout_s, errors.word(q.device), q_rot, wait_q, step_delta, epoch_per_step)
        return o, lse
    qf = q[:, : H * Dh].float().view(B, Sq, H, Dh)
    kf = k[:, : H * Dh].float().view(B, Skv, H, Dh)
    vf = v[:, : H * Dh].float().view(B, Skv, H, Dh)
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    l = torch.logsumexp(s, -1)
    p = torch.exp(s - l[..., None])
    of = torch.einsum("bhqk,bkhd->bqhd", p, vf)
    o.copy_(of.reshape(B * Sq, H * Dh).to(o.dtype))
    lse.view(B, H, -1)[:, :, :Sq].copy_(l)
    return o, lse


def attn_bwd(q, k, v, o, do, lse, B, Sq, Skv, H, Dh, scale=None, dk_out=None, dv_out=None, dq_out=None,
             push=None, delta=None):
    """Returns (dq [B*Sq,H*Dh] bf16, dk, dv [B*Skv, H*Dh] bf16).

    delta (optional): rowsum(dO * O) fp32 in the lse layout [B, H, lse_ld(Sq)],
    0 past Sq; when given, `o` is not read (may be None).

    push (CUDA, sequence parallel): dict(bases, chunk, rank, slot, ld, vcol):
    the keys are len(bases) chunks of `chunk` rows per sample; the kernel
    stores the dK/dV rows of chunk c straight into rank c's receive buffer
    (peer address bases[c], slot `rank` of `slot` elements, row stride `ld`,
    dV `vcol` columns after dK) and returns (dq, None, None)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(Dh)
    if push is not None:
        assert _cuda(q), "dK/dV push needs the CUDA kernels"
        dq = dq_out if dq_out is not None else torch.empty(B * Sq, H * Dh, device=q.device, dtype=q.dtype)
        delta = rowdot(do, o, H, Dh, Sq) if delta is None else delta
        dq_acc = torch.zeros(B * H * Sq * Dh, device=q.device)
        dummy = torch.empty(0, H * Dh, device=q.device, dtype=q.dtype)
        torch.ops.harp.attn_bwd(q, k, v, do, lse, delta, B, Sq, Skv, H, Dh, scale, dq_acc, dummy, dummy,
                                errors.word(q.device), push["bases"], push["chunk"], push["rank"], push["slot"],
                                push["ld"], push["vcol"])
        torch.ops.harp.dq_finalize(dq_acc, H, Dh, scale, dq, Sq)
        return dq, None, None
    dk = dk_out if dk_out is not None else torch.empty(B * Skv, H * Dh, device=q.device, dtype=q.dtype)
    dv = dv_out if dv_out is not None else torch.empty(B * Skv, H * Dh, device=q.device, dtype=q.dtype)
    dq = dq_out if dq_out is not None else torch.empty(B * Sq, H * Dh, device=q.device, dtype=q.dtype)
    if _cuda(q):
        delta = rowdot(do, o, H, Dh, Sq) if delta is None else delta
        dq_acc = torch.zeros(B * H * Sq * Dh, device=q.device)  # [B, H, Sq, Dh]
        torch.ops.harp.attn_bwd(q, k, v, do, lse, delta, B, Sq, Skv, H, Dh, scale, dq_acc, dk, dv,
                                errors.word(q.device))
        torch.ops.harp.dq_finalize(dq_acc, H, Dh, scale, dq, Sq)
        return dq, dk, dv
    qf = q[:, : H * Dh].float().view(B, Sq, H, Dh)
    kf = k[:, : H * Dh].float().view(B, Skv, H, Dh)
    vf = v[:, : H * Dh].float().view(B, Skv, H, Dh)
    dof = do.float().view(B, Sq, H, Dh)
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    p = torch.exp(s - lse.view(B, H, -1)[:, :, :Sq, None])
    dvf = torch.einsum("bhqk,bqhd->bkhd", p, dof)
    dp = torch.einsum("bqhd,bkhd->bhqk", dof, vf)
    if delta is None:
        delta = (dof * o.float().view(B, Sq, H, Dh)).sum(-1).permute(0, 2, 1)[..., None]
    else:
        delta = delta.view(B, H, -1)[:, :, :Sq, None].float()
    ds = p * (dp - delta)
    dqf = torch.einsum("bhqk,bkhd->bqhd", ds, kf) * scale
    dkf = torch.einsum("bhqk,bqhd->bkhd", ds, qf) * scale
    dq.copy_(dqf.reshape(B * Sq, H * Dh).to(dq.dtype))
    dk.copy_(dkf.reshape(B * Skv, H * Dh).to(dk.dtype))
    dv.copy_(dvf.reshape(B * Skv, H * Dh).to(dv.dtype))
    return dq, dk, dv


# ---------------------------------------------------------------------------
# optimizer
# ---------------------------------------------------------------------------
def adamw_flat(master, m, v, grad, param, lr, beta1, beta2, eps, wd, step, grad_scale=1.0, hyper=None):
    """AdamW on flat fp32 state.  `hyper` (CUDA only): fp32 device tensor
    [lr, 1 - beta1^step, sqrt(1 - beta2^step)] read at run time instead of
    `lr` / `step` (CUDA-graph replays)."""
    if _cuda(master):
        torch.ops.harp.adamw_flat(master, m, v, grad, param, lr, beta1, beta2, eps, wd, step, grad_scale, hyper)
        return
    g = grad.float() * grad_scale
    master.mul_(1 - lr * wd)
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    master.addcdiv_(m, denom, value=-lr / bc1)
    if param is not None:
        param.copy_(master.to(param.dtype))


def philox_uniform_(t: torch.Tensor, seed: int, offset: int, lo: float, hi: float) -> torch.Tensor:
    """Fill with U[lo, hi) from Philox4x32-10 (same stream on every rank for a seed)."""
    if _cuda(t):
        torch.ops.harp.philox_uniform(t, seed, offset, lo, hi)
        return t
    g = torch.Generator().manual_seed((seed * 1000003 + offset) & 0x7FFFFFFFFFFFFFFF)
    t.copy_(torch.rand(t.shape, generator=g) * (hi - lo) + lo)
    return t
