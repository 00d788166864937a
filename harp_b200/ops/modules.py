"""Autograd ops and nn.Modules over the harp kernels (op layer).

These serve the model families that run op by op (Z-Image, MMDiT, Flux); the
flagship DiT runs its block as one fused autograd function (models/dit.py).

Reference op layer (L3) and the names kept for it:
  kpLinear / CustomLinearFunction / replace_linear_with_kplinear
                                   unigemm_linear.py:8-108 (xhpops::kp_linear_*)
  kpRMSNorm / replace_rmsNorm_with_kpRMSNorm   kp_normalization.py:8-99
  MySiLU, MyTanh, ApplyRotaryComplexFn         async_rt/async_ops.py:125-178
  kp_multi_tensor_adamw                        kp_multi_tensor_adamw.py:7-69
Each one calls the harp CUDA kernel on GPU tensors and the fp32 restatement on
CPU tensors (harp_b200.ops.functional).
"""
from __future__ import annotations

import math
import numbers
from typing import List, Optional

import torch
import torch.nn as nn

from . import functional as Fn
from ..parallel.sequence import SPContext, sp_attention_backward, sp_attention_forward


# ---------------------------------------------------------------------------
# Linear
# ---------------------------------------------------------------------------
class LinearFunction(torch.autograd.Function):
    """y = x W^T + b on the harp GEMM (any leading dims)."""

    @staticmethod
    def forward(ctx, x, w, b):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.dtype != w.dtype:
            x2 = x2.to(w.dtype)
        y = Fn.gemm(x2, w, bias=b)
        ctx.save_for_backward(x2, w)
        ctx.has_b = b is not None
        ctx.shp = shp
        ctx.in_dtype = x.dtype
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(w.dtype).contiguous()
        dx, dw, db = Fn.linear_bwd(dy2, x2, w, need_bias=ctx.has_b)
        return dx.view(ctx.shp).to(ctx.in_dtype), dw, (db.to(w.dtype) if db is not None else None)


CustomLinearFunction = LinearFunction


def linear(x, w, b=None):
    return LinearFunction.apply(x, w, b)


class kpLinear(nn.Module):
    """bf16 linear layer on the harp GEMM; same parameter names as nn.Linear."""

    def __init__(self, in_features, out_features, bias=True, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.empty(out_features, device=device, dtype=dtype)) if bias else None
        self.reset_parameters()

    def reset_parameters(self):
        w = torch.empty(self.weight.shape, dtype=torch.float32)
        nn.init.kaiming_uniform_(w, a=math.sqrt(5))
        self.weight.data.copy_(w.to(self.weight.dtype))
        if self.bias is not None:
            bound = 1 / math.sqrt(self.in_features) if self.in_features > 0 else 0
            self.bias.data.copy_(torch.empty(self.bias.shape).uniform_(-bound, bound).to(self.bias.dtype))

    def forward(self, x):
        return LinearFunction.apply(x, self.weight, self.bias)


def replace_linear_with_kplinear(model: nn.Module, kplinear_class=kpLinear) -> nn.Module:
    for name, child in list(model.named_children()):
        if isinstance(child, nn.Linear):
            new = kplinear_class(child.in_features, child.out_features, bias=child.bias is not None,
                                 device=child.weight.device)
            new.weight.data.copy_(child.weight.data)
            if child.bias is not None:
                new.bias.data.copy_(child.bias.data)
            setattr(model, name, new)
        else:
            replace_linear_with_kplinear(child, kplinear_class)
    return model


# ---------------------------------------------------------------------------
# RMSNorm (optional affine weight)
# ---------------------------------------------------------------------------
class RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, rstd = Fn.rmsnorm_mod_fwd(x2, w, None, None, x2.shape[0], eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shp = shp
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).contiguous()
        dx, dw, _, _ = Fn.rmsnorm_mod_bwd(x2, rstd, dy2, w, None, x2.shape[0], want_dw=w is not None)
        return dx.view(ctx.shp), (dw.to(w.dtype) if dw is not None else None), None


class kpRMSNorm(nn.Module):
    def __init__(self, dim, eps: float = 1e-6, elementwise_affine: bool = True, bias: bool = False,
                 device=None, dtype=None):
        super().__init__()
        if bias:
            raise NotImplementedError("RMSNorm bias is not supported")
        self.dim = torch.Size((dim,) if isinstance(dim, numbers.Integral) else dim)
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        self.weight = nn.Parameter(torch.ones(self.dim, device=device, dtype=dtype)) if elementwise_affine else None

    def forward(self, x):
        if x.shape[-1] % 8 != 0:  # the kernels vectorize by 8
            xf = x.float()
            y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
            return (y * self.weight.float() if self.weight is not None else y).to(x.dtype)
        return RMSNormFunction.apply(x, self.weight, self.eps)


RMSNorm = kpRMSNorm
CustomNormFunction = RMSNormFunction  # the reference's name (kp_normalization.py:8)


def _is_rmsnorm(m: nn.Module) -> bool:
    return isinstance(m, nn.RMSNorm) or type(m).__name__ == "RMSNorm"


def replace_rmsNorm_with_kpRMSNorm(module: nn.Module) -> nn.Module:
    for name, child in list(module.named_children()):
        if _is_rmsnorm(child) and not isinstance(child, kpRMSNorm):
            dim = getattr(child, "dim", None) or getattr(child, "normalized_shape", None)
            eps = getattr(child, "eps", None) or 1e-6
            w = getattr(child, "weight", None)
            new = kpRMSNorm(tuple(dim), eps=eps, elementwise_affine=w is not None,
                            device=w.device if w is not None else None, dtype=w.dtype if w is not None else None)
            if w is not None:
                new.weight.data.copy_(w.data)
                new.weight.requires_grad_(w.requires_grad)
            setattr(module, name, new)
        else:
            replace_rmsNorm_with_kpRMSNorm(child)
    return module


# ---------------------------------------------------------------------------
# elementwise
# ---------------------------------------------------------------------------
class MySiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        ctx.save_for_backward(x)
        return Fn.silu(x)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return Fn.silu_bwd(dy.contiguous(), x)


SiLUFunction = MySiLU


class MyTanh(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        if x.is_cuda and x.dtype == torch.bfloat16:
            y = torch.empty_like(x)
            torch.ops.async_op.tanh_out(x, y)
        else:
            y = torch.tanh(x.float()).to(x.dtype)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, dy):
        (y,) = ctx.saved_tensors
        if y.is_cuda and y.dtype == torch.bfloat16:
            dx = torch.empty_like(y)
            torch.ops.async_op.tanh_backward_out(dy.contiguous(), y, dx)
            return dx
        return (dy.float() * (1 - y.float() ** 2)).to(y.dtype)


# ---------------------------------------------------------------------------
# QK RMSNorm + RoPE on token-major [B, S, H*Dh] q and k
# ---------------------------------------------------------------------------
class QKNormRopeFunction(torch.autograd.Function):
    """(q, k) -> (rope(rms_h(q)*wq), rope(rms_h(k)*wk)); freqs fp32 [F, Dh/2, 2]
    (cos, sin) with token row r using freqs[r % F]; norm weights may be None."""

    @staticmethod
    def forward(ctx, q, k, wq, wk, freqs, H, Dh, eps, do_norm):
        shp = q.shape
        R = q.numel() // (H * Dh)
        qk = torch.cat([q.reshape(R, H * Dh), k.reshape(R, H * Dh)], 1)
        qo, ko, rq, rk = Fn.qknorm_rope_fwd(qk, H, Dh, wq, wk, freqs, eps, do_norm=do_norm)
        ctx.save_for_backward(qk, rq if do_norm else qk.new_empty(0), rk if do_norm else qk.new_empty(0), freqs,
                              wq if wq is not None else qk.new_empty(0), wk if wk is not None else qk.new_empty(0))
        ctx.meta = (shp, H, Dh, do_norm, wq is not None)
        return qo.view(shp), ko.view(shp)

    @staticmethod
    def backward(ctx, dq, dk):
        qk, rq, rk, freqs, wq, wk = ctx.saved_tensors
        shp, H, Dh, do_norm, has_w = ctx.meta
        R = qk.shape[0]
        dqk = torch.empty_like(qk)
        dwq, dwk = Fn.qknorm_rope_bwd(dq.reshape(R, H * Dh).contiguous(), dk.reshape(R, H * Dh).contiguous(), qk,
                                      rq if do_norm else None, rk if do_norm else None, H, Dh,
                                      wq if has_w else None, wk if has_w else None, freqs, do_norm, dqk,
                                      want_dw=has_w and do_norm)
        return (dqk[:, : H * Dh].reshape(shp), dqk[:, H * Dh:].reshape(shp),
                dwq.to(wq.dtype) if dwq is not None else None, dwk.to(wk.dtype) if dwk is not None else None,
                None, None, None, None, None)


def complex_to_freqs(freqs_cis: torch.Tensor) -> torch.Tensor:
    """complex64 [..., Dh/2] (cos + i sin) -> fp32 [N, Dh/2, 2] with N = prod(leading dims)."""
    f = torch.view_as_real(freqs_cis.to(torch.complex64))
    return f.reshape(-1, f.shape[-2], 2).contiguous()


class ApplyRotaryComplexFn(torch.autograd.Function):
    """x * freqs_cis over interleaved complex pairs (async_op::rope_forward_impl).
    x: [B, H, T, D] (a view of token-major [B, T, H*D] storage, as the reference
    builds it) or [B, T, H, D]; freqs_cis: complex [B, T, D/2] or [T, D/2]."""

    @staticmethod
    def forward(ctx, x, freqs_cis):
        ctx.save_for_backward(freqs_cis)
        return _rope_apply(x, freqs_cis, inverse=False)

    @staticmethod
    def backward(ctx, g):
        (freqs_cis,) = ctx.saved_tensors
        return _rope_apply(g, freqs_cis, inverse=True), None


def kp_apply_rotary_emb(x, freqs_cis, use_real: bool = True, use_real_unbind_dim: int = -1):
    """Rotary embedding of x [B, H, S, D] by complex freqs_cis (kp_rope.py:4-14);
    as in the reference only the complex form (use_real=False) exists."""
    if use_real:
        raise NotImplementedError("kp_apply_rotary_emb: only the complex form (use_real=False)")
    return ApplyRotaryComplexFn.apply(x, freqs_cis)


def _rope_apply(x, freqs_cis, inverse):
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    f = torch.view_as_real(freqs_cis.to(torch.complex64))
    c, s = f[..., 0], f[..., 1]
    if x.dim() == 4 and freqs_cis.dim() == 3 and x.shape[2] == freqs_cis.shape[1]:
        c, s = c[:, None], s[:, None]  # [B, 1, T, D/2] against x [B, H, T, D]
    elif x.dim() == 4 and freqs_cis.dim() == 2:
        c, s = c[None, None], s[None, None]
    x0, x1 = xf[..., 0], xf[..., 1]
    if inverse:
        o0, o1 = x0 * c + x1 * s, -x0 * s + x1 * c
    else:
        o0, o1 = x0 * c - x1 * s, x0 * s + x1 * c
    return torch.stack([o0, o1], -1).reshape(x.shape).to(x.dtype)


# ---------------------------------------------------------------------------
# attention over the (sequence-parallel) sequence
# ---------------------------------------------------------------------------
class SPAttentionFunction(torch.autograd.Function):
    """softmax(q k^T / sqrt(Dh)) v over all SP chunks; q, k, v: [B, S_local, H*Dh]."""

    @staticmethod
    def forward(ctx, q, k, v, H, Dh, sp):
        B, S, _ = q.shape
        q2, k2, v2 = (t.reshape(B * S, H * Dh).contiguous() for t in (q, k, v))
        o, saved = sp_attention_forward(q2, k2, v2, B, S, H, Dh, sp)
        ctx.save_for_backward(q2, k2, v2, o)
        ctx.saved = saved
        ctx.meta = (B, S, H, Dh, sp)
        return o.view(B, S, H * Dh)

    @staticmethod
    def backward(ctx, do):
        q2, k2, v2, o = ctx.saved_tensors
        B, S, H, Dh, sp = ctx.meta
        dq, dk, dv = sp_attention_backward(ctx.saved, q2, k2, v2, o, do.reshape(B * S, H * Dh).contiguous(), B, S,
                                           H, Dh, sp)
        shp = (B, S, H * Dh)
        return dq.view(shp), dk.contiguous().view(shp), dv.contiguous().view(shp), None, None, None


def sp_attention(q, k, v, heads: int, head_dim: int, sp: Optional[SPContext] = None):
    return SPAttentionFunction.apply(q, k, v, heads, head_dim, sp or SPContext())


# ---------------------------------------------------------------------------
# multi-tensor AdamW (reference kp_multi_tensor_adamw: no weight decay was
# passed there; here it is honoured)
# ---------------------------------------------------------------------------
def kp_multi_tensor_adamw(params: List[torch.Tensor], grads: List[torch.Tensor], exp_avgs: List[torch.Tensor],
                          exp_avg_sqs: List[torch.Tensor], max_exp_avg_sqs, state_steps: List[torch.Tensor],
                          grad_scale=None, found_inf=None, *, amsgrad: bool, beta1: float, beta2: float, lr,
                          weight_decay: float, eps: float, maximize: bool, capturable: bool, differentiable: bool,
                          has_complex: bool):
    """Drop-in for torch.optim.adamw._multi_tensor_adamw on CUDA tensors
    (one launch over every tensor), torch's own update elsewhere."""
    if not params:
        return
    assert not amsgrad and not maximize and grad_scale is None and found_inf is None
    lr = float(lr)
    if params[0].is_cuda:
        torch.ops.async_op.foreach_adamw_wd(params, grads, exp_avgs, exp_avg_sqs, state_steps, beta1, beta2, eps, lr,
                                            weight_decay)
        return
    for p, g, m, v, st in zip(params, grads, exp_avgs, exp_avg_sqs, state_steps):
        st += 1
        step = int(st.item())
        p.mul_(1 - lr * weight_decay)
        m.mul_(beta1).add_(g, alpha=1 - beta1)
        v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
        denom = (v.sqrt() / math.sqrt(1 - beta2 ** step)).add_(eps)
        p.addcdiv_(m, denom, value=-lr / (1 - beta1 ** step))


def install_multi_tensor_adamw():
    """Route torch.optim.AdamW(foreach=True) through the harp kernel, as the
    reference patches adamw._multi_tensor_adamw (train.py:43-45)."""
    import torch.optim.adamw as adamw_mod

    adamw_mod._multi_tensor_adamw = kp_multi_tensor_adamw
