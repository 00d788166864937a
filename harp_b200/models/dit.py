"""Generic DiT (adaLN-zero, RMSNorm, 3-axis RoPE, QK-RMSNorm, SwiGLU) with a
fused, hand-scheduled transformer block.

The reference trains one model family, Z-Image (src/models/z_image/
standalone_transformer.py:294-355 for the block); the benchmark configurations
of this framework name a DiT-XL/2-style model, an MMDiT and a Flux-like model.
This file is the DiT: joint self-attention over [image tokens ; text tokens],
conditioning by adaLN-zero on the timestep embedding.

``DiTBlockFunction`` runs the whole block as one autograd node:

  forward                                        kernels
    mod   = Linear(silu(c))      [B, 6D]         harp gemm (M = B)
    h1    = rms(x)*(1+sc1)+sh1                   rmsnorm_mod_fwd
    qkv   = h1 Wqkv^T + b                        gemm
    q,k   = rope(rms_h(q)*wq), rope(rms_h(k)*wk) qknorm_rope_fwd
    o     = attention(q, k, v)  (ring over SP)   attn_fwd (+ NVLink KV exchange)
    x1    = x + g1 * (o Wo^T + bo)               gemm, gated-residual epilogue
    h2    = rms(x1)*(1+sc2)+sh2                  rmsnorm_mod_fwd
    gu    = h2 [W1;W3]^T                         gemm (w1, w3 adjacent in memory)
    hh    = silu(g)*u                            swiglu_fwd
    x2    = x1 + g2 * (hh W2^T + b2)             gemm, gated-residual epilogue
  backward mirrors it with gate_bwd, swiglu_bwd, rmsnorm_mod_bwd (with the
  residual gradient folded in), qknorm_rope_bwd, attn_bwd and the dX / dW GEMMs.

On CPU the same function runs on the fp32 restatements of each op (the oracle
used by the tests).
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from ..ops import functional as Fn
from ..ops.modules import LinearFunction, SiLUFunction
from ..parallel.sequence import SPContext, qkv_attention_backward, qkv_attention_forward


# ---------------------------------------------------------------------------
# configuration
# ---------------------------------------------------------------------------
@dataclass
class DiTConfig:
    in_channels: int = 16
    patch_size: int = 2
    hidden: int = 1152
    depth: int = 28
    heads: int = 16
    mlp_ratio: float = 4.0
    text_dim: int = 1152
    qk_norm: bool = True
    norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    axes_dims: Tuple[int, int, int] = (24, 24, 24)
    learn_sigma: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def ffn_hidden(self) -> int:
        return int(self.hidden * self.mlp_ratio)

    @property
    def patch_dim(self) -> int:
        return self.patch_size * self.patch_size * self.in_channels

    def to_dict(self):
        d = asdict(self)
        d["axes_dims"] = list(self.axes_dims)
        return d


PRESETS = {
    # DiT-XL/2 at 1024px (latent 128x128, 4096 image tokens + 256 text tokens)
    "dit-xl-2": DiTConfig(hidden=1152, depth=28, heads=16, mlp_ratio=4.0, text_dim=1152, axes_dims=(24, 24, 24)),
    # ~2.3B joint-attention DiT (Lumina-style: image and text tokens share every
    # block's weights), 24 blocks, hidden 2304, 18 heads x 128, SwiGLU 6144
    "mmdit-2b": DiTConfig(hidden=2304, depth=24, heads=18, mlp_ratio=8.0 / 3.0, text_dim=2304,
                          axes_dims=(32, 48, 48)),
    # tiny DiT for CPU/gloo plumbing tests
    "tiny": DiTConfig(in_channels=4, hidden=384, depth=6, heads=6, mlp_ratio=4.0, text_dim=384,
                      axes_dims=(16, 24, 24)),
    # a few-layer variant used by GPU smoke tests
    "small": DiTConfig(in_channels=16, hidden=384, depth=2, heads=6, mlp_ratio=4.0, text_dim=384,
                       axes_dims=(16, 24, 24)),
}


# ---------------------------------------------------------------------------
# RoPE tables
# ---------------------------------------------------------------------------
def rope_freqs(positions: torch.Tensor, axes_dims: Sequence[int], theta: float) -> torch.Tensor:
    """positions: int [N, n_axes] -> fp32 [N, sum(axes)/2, 2] (cos, sin) per
    complex pair; pairs of axis a use frequencies theta^(-2i/d_a)."""
    parts = []
    for a, d in enumerate(axes_dims):
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
        ang = positions[:, a].double()[:, None] * inv[None, :]
        parts.append(ang)
    ang = torch.cat(parts, -1)
    return torch.stack([ang.cos(), ang.sin()], -1).float().contiguous()


def joint_positions(h_tokens: int, w_tokens: int, text_len: int) -> torch.Tensor:
    """Image tokens (row-major h, w) first, then text tokens.  Axis 0 separates
    the streams (image at text_len+1, text at 1..text_len), axes 1-2 carry the
    2-D image position."""
    hh, ww = torch.meshgrid(torch.arange(h_tokens), torch.arange(w_tokens), indexing="ij")
    img = torch.stack([torch.full_like(hh, text_len + 1), hh, ww], -1).reshape(-1, 3)
    txt = torch.stack([torch.arange(1, text_len + 1), torch.zeros(text_len, dtype=torch.long),
                       torch.zeros(text_len, dtype=torch.long)], -1)
    return torch.cat([img, txt], 0)


# ---------------------------------------------------------------------------
# modules (parameter holders; names give the state_dict layout)
# ---------------------------------------------------------------------------
class _Linear(nn.Module):
    def __init__(self, in_f, out_f, bias=True, weight: Optional[torch.Tensor] = None):
        super().__init__()
        self.in_features, self.out_features = in_f, out_f
        self.weight = nn.Parameter(weight if weight is not None else torch.empty(out_f, in_f))
        self.bias = nn.Parameter(torch.zeros(out_f)) if bias else None


class _RMSWeight(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class Attention(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        D = cfg.hidden
        self.qkv = _Linear(D, 3 * D, bias=True)
        self.q_norm = _RMSWeight(cfg.head_dim, 1e-6) if cfg.qk_norm else None
        self.k_norm = _RMSWeight(cfg.head_dim, 1e-6) if cfg.qk_norm else None
        self.proj = _Linear(D, D, bias=True)


class SwiGLU(nn.Module):
    """w1 and w3 are views of one [2F, D] buffer so the up projection is a single GEMM."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        w13 = torch.empty(2 * F_, D)
        self.w1 = _Linear(D, F_, bias=False, weight=w13[:F_])
        self.w3 = _Linear(D, F_, bias=False, weight=w13[F_:])
        self.w2 = _Linear(F_, D, bias=True)


class DiTBlock(nn.Module):
    def __init__(self, cfg: DiTConfig, layer_id: int):
        super().__init__()
        self.cfg = cfg
        self.layer_id = layer_id
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), _Linear(cfg.hidden, 6 * cfg.hidden, bias=True))
        self.attn = Attention(cfg)
        self.mlp = SwiGLU(cfg)

    def block_params(self) -> List[torch.Tensor]:
        a, m = self.attn, self.mlp
        ps = [self.adaLN_modulation[1].weight, self.adaLN_modulation[1].bias, a.qkv.weight, a.qkv.bias]
        ps += [a.q_norm.weight if a.q_norm is not None else None, a.k_norm.weight if a.k_norm is not None else None]
        ps += [a.proj.weight, a.proj.bias, m.w1.weight, m.w3.weight, m.w2.weight, m.w2.bias]
        return ps

    def forward(self, x: torch.Tensor, c_silu: torch.Tensor, freqs: torch.Tensor, sp: SPContext) -> torch.Tensor:
        ps = self.block_params()
        live = [p for p in ps if p is not None]
        return DiTBlockFunction.apply(x, c_silu, freqs, self, sp, *live)


def _w13(w1: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """[W1; W3] without a copy when w3 directly follows w1 in memory."""
    F_, D = w1.shape
    if (w1.is_contiguous() and w3.is_contiguous() and w1.untyped_storage().data_ptr() ==
            w3.untyped_storage().data_ptr() and w3.data_ptr() == w1.data_ptr() + w1.numel() * w1.element_size()):
        return torch.as_strided(w1, (2 * F_, D), (D, 1))
    return torch.cat([w1, w3], 0)


class DiTBlockFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, c_silu, freqs, blk: DiTBlock, sp: SPContext, *params):
        cfg = blk.cfg
        B, S, D = x.shape
        H, Dh, F_ = cfg.heads, cfg.head_dim, cfg.ffn_hidden
        R = B * S
        ps = blk.block_params()
        ada_w, ada_b, qkv_w, qkv_b, qn_w, kn_w, proj_w, proj_b, w1, w3, w2, w2_b = ps
        x2d = x.reshape(R, D)

        mod = Fn.gemm(c_silu, ada_w, bias=ada_b)  # [B, 6D]
        sh1, sc1, g1, sh2, sc2, g2 = (mod[:, i * D:(i + 1) * D] for i in range(6))
        h1, rstd1 = Fn.rmsnorm_mod_fwd(x2d, None, sc1, sh1, S, cfg.norm_eps)
        qkv = Fn.gemm(h1, qkv_w, bias=qkv_b)  # [R, 3D]
        o, rq, rk, q, k, attn_saved = qkv_attention_forward(qkv, B, S, H, Dh, qn_w, kn_w, freqs, 1e-6, cfg.qk_norm,
                                                            sp)
        a1 = torch.empty(R, D, device=x.device, dtype=x.dtype)
        x1 = Fn.gemm(o, proj_w, bias=proj_b, epi=Fn.EPI_GATED_RESIDUAL_SAVE, residual=x2d, gate=g1,
                     rows_per_batch=S, out2=a1)
        h2, rstd2 = Fn.rmsnorm_mod_fwd(x1, None, sc2, sh2, S, cfg.norm_eps)
        gu = Fn.gemm(h2, _w13(w1, w3))  # [R, 2F]
        hh = Fn.swiglu_fwd(gu, F_)
        a2 = torch.empty(R, D, device=x.device, dtype=x.dtype)
        x2 = Fn.gemm(hh, w2, bias=w2_b, epi=Fn.EPI_GATED_RESIDUAL_SAVE, residual=x1, gate=g2, rows_per_batch=S,
                     out2=a2)

        ctx.blk, ctx.sp = blk, sp
        ctx.shape = (B, S, D)
        ctx.attn_saved = attn_saved
        ctx.save_for_backward(x2d, c_silu, freqs, mod, h1, rstd1, qkv, q, k, rq, rk, o, a1, x1, rstd2, h2, gu, hh,
                              a2)
        return x2.view(B, S, D)

    @staticmethod
    def backward(ctx, dy):
        blk, sp = ctx.blk, ctx.sp
        cfg = blk.cfg
        B, S, D = ctx.shape
        H, Dh, F_ = cfg.heads, cfg.head_dim, cfg.ffn_hidden
        R = B * S
        (x2d, c_silu, freqs, mod, h1, rstd1, qkv, q, k, rq, rk, o, a1, x1, rstd2, h2, gu, hh,
         a2) = ctx.saved_tensors
        ps = blk.block_params()
        ada_w, ada_b, qkv_w, qkv_b, qn_w, kn_w, proj_w, proj_b, w1, w3, w2, w2_b = ps
        sh1, sc1, g1, sh2, sc2, g2 = (mod[:, i * D:(i + 1) * D] for i in range(6))
        dy = dy.reshape(R, D).contiguous()
        dmod = torch.empty(B, 6 * D, device=dy.device, dtype=torch.float32)

        # ---- MLP branch: x2 = x1 + g2 * (hh W2^T + b2)
        da2, dg2, db2 = Fn.gate_bwd(dy, a2, g2, S, want_bias=True)
        dmod[:, 5 * D:6 * D] = dg2
        dhh, dw2, _ = Fn.linear_bwd(da2, hh, w2, need_bias=False, dw_out=_direct(w2))
        dgu = Fn.swiglu_bwd(dhh, gu)
        w13 = _w13(w1, w3)
        g1d, g3d = _direct(w1), _direct(w3)
        dw13_out = _w13(g1d, g3d) if (g1d is not None and g3d is not None) else None
        if dw13_out is not None and dw13_out.data_ptr() != g1d.data_ptr():
            dw13_out = None  # the two slots are not adjacent: write to a temporary instead
        dh2, dw13, _ = Fn.linear_bwd(dgu, h2, w13, need_bias=False, dw_out=dw13_out)
        dx1, _, dsc2, dsh2 = Fn.rmsnorm_mod_bwd(x1, rstd2, dh2, None, sc2, S, dres=dy, want_mod=True)
        dmod[:, 3 * D:4 * D] = dsh2
        dmod[:, 4 * D:5 * D] = dsc2

        # ---- attention branch: x1 = x + g1 * (o Wo^T + bo)
        da1, dg1, dbo = Fn.gate_bwd(dx1, a1, g1, S, want_bias=True)
        dmod[:, 2 * D:3 * D] = dg1
        do, dwo, _ = Fn.linear_bwd(da1, o, proj_w, need_bias=False, dw_out=_direct(proj_w))
        dqkv, dwq, dwk = qkv_attention_backward(ctx.attn_saved, qkv, q, k, o, do, rq, rk, qn_w, kn_w, freqs,
                                                cfg.qk_norm, B, S, H, Dh, sp)
        dh1, dwqkv, dbqkv = Fn.linear_bwd(dqkv, h1, qkv_w, need_bias=True, dw_out=_direct(qkv_w))
        dx, _, dsc1, dsh1 = Fn.rmsnorm_mod_bwd(x2d, rstd1, dh1, None, sc1, S, dres=dx1, want_mod=True)
        dmod[:, 0:D] = dsh1
        dmod[:, D:2 * D] = dsc1

        # ---- adaLN: mod = silu(c) W^T + b
        dmod_b = dmod.to(torch.bfloat16)
        dada_w = Fn.gemm(dmod_b, c_silu, a_mn=True, b_mn=True, out=_direct(ada_w))  # [6D, Dc]
        dada_b = dmod.sum(0)
        dc_silu = Fn.gemm(dmod_b, ada_w, b_mn=True)  # [B, Dc]

        grads = [_emit(ada_w, dada_w), _emit(ada_b, dada_b), _emit(qkv_w, dwqkv), _emit(qkv_b, dbqkv)]
        if cfg.qk_norm:
            grads += [_emit(qn_w, dwq), _emit(kn_w, dwk)]
        grads += [_emit(proj_w, dwo), _emit(proj_b, dbo), _emit(w1, dw13[:F_]), _emit(w3, dw13[F_:]),
                  _emit(w2, dw2), _emit(w2_b, db2)]
        return (dx.view(B, S, D), dc_silu, None, None, None, *grads)


def _direct(p: torch.Tensor) -> Optional[torch.Tensor]:
    """The gradient slot of `p` when the trainer enabled direct gradient writes
    (p.grad is then a view into the flat gradient buffer, zeroed every step).
    The fused block uses each of its parameters exactly once per step, so its
    weight-gradient GEMMs can store straight into that slot."""
    if getattr(p, "_harp_direct_grad", False) and p.grad is not None:
        return p.grad
    return None


def _emit(p: torch.Tensor, g: torch.Tensor):
    """What backward returns for parameter `p`: None when the gradient went
    (or now goes) straight into p's slot, else the gradient in p's dtype."""
    tgt = _direct(p)
    if tgt is None:
        return g.to(p.dtype)
    if g.data_ptr() != tgt.data_ptr():
        tgt.copy_(g.view_as(tgt))
    # the slot now holds this step's complete gradient (enqueued on the current
    # stream): tell the trainer, which may send the bucket that holds it
    cb = getattr(p, "_harp_grad_ready", None)
    if cb is not None:
        cb(p)
    return None


# ---------------------------------------------------------------------------
# embedders / final layer
# ---------------------------------------------------------------------------
class TimestepEmbedder(nn.Module):
    """Sinusoidal (cos, sin) embedding followed by Linear-SiLU-Linear, as the
    reference's TimestepEmbedder (src/models/embedding.py:136-158)."""

    def __init__(self, out_size, mid_size=None, freq_dim=256):
        super().__init__()
        mid_size = mid_size or out_size
        self.freq_dim = freq_dim
        self.mlp = nn.Sequential(_Linear(freq_dim, mid_size), nn.SiLU(), _Linear(mid_size, out_size))

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        args = t[:, None].float() * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], -1)

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        f = self.timestep_embedding(t, self.freq_dim).to(self.mlp[0].weight.dtype)
        h = LinearFunction.apply(f, self.mlp[0].weight, self.mlp[0].bias)
        h = SiLUFunction.apply(h)
        return LinearFunction.apply(h, self.mlp[2].weight, self.mlp[2].bias)


class FinalLayerFunction(torch.autograd.Function):
    """out = (LN(x)*(1+scale)+shift) W^T + b, with (shift, scale) = Linear(silu(c))."""

    @staticmethod
    def forward(ctx, x, c_silu, ada_w, ada_b, w, b):
        B, S, D = x.shape
        x2 = x.reshape(B * S, D)
        mod = Fn.gemm(c_silu, ada_w, bias=ada_b)  # [B, 2D] = shift, scale
        shift, scale = mod[:, :D], mod[:, D:]
        y, mean, rstd = Fn.layernorm_mod_fwd(x2, scale, shift, S, 1e-6)
        out = Fn.gemm(y, w, bias=b)
        ctx.save_for_backward(x2, c_silu, mod, y, mean, rstd, ada_w, w)
        ctx.shape = (B, S, D)
        return out.view(B, S, -1)

    @staticmethod
    def backward(ctx, dout):
        x2, c_silu, mod, y, mean, rstd, ada_w, w = ctx.saved_tensors
        B, S, D = ctx.shape
        dout2 = dout.reshape(B * S, -1).contiguous()
        dy, dw, db = Fn.linear_bwd(dout2, y, w, need_bias=True)
        dx, dscale, dshift = Fn.layernorm_mod_bwd(x2, mean, rstd, dy, mod[:, D:], S, want_mod=True)
        dmod = torch.cat([dshift, dscale], 1)
        dmod_b = dmod.to(torch.bfloat16)
        dada_w = Fn.gemm(dmod_b, c_silu, a_mn=True, b_mn=True)
        dada_b = dmod.sum(0).to(torch.bfloat16)
        dc = Fn.gemm(dmod_b, ada_w, b_mn=True)
        return dx.view(B, S, D), dc, dada_w, dada_b, dw, db.to(w.dtype)


class FinalLayer(nn.Module):
    def __init__(self, hidden, out_dim):
        super().__init__()
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), _Linear(hidden, 2 * hidden))
        self.linear = _Linear(hidden, out_dim)

    def forward(self, x, c_silu):
        return FinalLayerFunction.apply(x, c_silu, self.adaLN_modulation[1].weight, self.adaLN_modulation[1].bias,
                                        self.linear.weight, self.linear.bias)


# ---------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------
class DiT(nn.Module):
    """Sequence-parallel DiT.  Each SP rank holds ``S_total / sp`` consecutive
    positions of the joint sequence [image tokens ; text tokens] and computes
    the loss on the image tokens it holds; every weight is replicated and its
    gradient is summed over all ranks by the gradient manager."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        D = cfg.hidden
        self.x_embedder = _Linear(cfg.patch_dim, D)
        self.t_embedder = TimestepEmbedder(D, mid_size=D)
        self.text_embedder = _Linear(cfg.text_dim, D)
        self.blocks = nn.ModuleList([DiTBlock(cfg, i) for i in range(cfg.depth)])
        self.final_layer = FinalLayer(D, cfg.patch_dim * (2 if cfg.learn_sigma else 1))
        self._freq_cache = {}

    # -- init -------------------------------------------------------------
    @torch.no_grad()
    def initialize_weights(self, seed: int = 0):
        """Xavier-uniform linears, zero adaLN (adaLN-zero), unit norm weights.
        Draws come from Philox keyed by parameter index, so every rank (and
        any device) builds identical weights, as the reference's shared-weight
        scheme requires (train.py:274-285)."""
        for i, (name, p) in enumerate(self.named_parameters()):
            if name.endswith("bias"):
                p.zero_()
            elif "norm" in name:
                p.fill_(1.0)
            elif "adaLN_modulation" in name:
                p.zero_()
            else:
                fan_out, fan_in = p.shape[0], p.shape[1]
                bound = math.sqrt(6.0 / (fan_in + fan_out))
                Fn.philox_uniform_(p.data, seed, i << 32, -bound, bound)
        # keep the output projection small but non-zero so gradients reach every block
        bound = 1e-3
        Fn.philox_uniform_(self.final_layer.linear.weight.data, seed, 0xFFFF << 32, -bound, bound)

    # -- helpers ------------------------------------------------------------
    def patchify(self, latent: torch.Tensor) -> torch.Tensor:
        B, C, Hh, Ww = latent.shape
        p = self.cfg.patch_size
        x = latent.view(B, C, Hh // p, p, Ww // p, p).permute(0, 2, 4, 3, 5, 1)
        return x.reshape(B, (Hh // p) * (Ww // p), p * p * C)

    def unpatchify(self, x: torch.Tensor, Hh: int, Ww: int) -> torch.Tensor:
        B, N, _ = x.shape
        p, C = self.cfg.patch_size, self.cfg.in_channels
        x = x.view(B, Hh // p, Ww // p, p, p, C).permute(0, 5, 1, 3, 2, 4)
        return x.reshape(B, C, Hh, Ww)

    def local_range(self, s_total: int, sp: SPContext) -> Tuple[int, int]:
        assert s_total % sp.size == 0, f"sequence {s_total} not divisible by sp {sp.size}"
        n = s_total // sp.size
        return sp.rank * n, (sp.rank + 1) * n

    def freqs_for(self, h_tok: int, w_tok: int, text_len: int, lo: int, hi: int, device) -> torch.Tensor:
        key = (h_tok, w_tok, text_len, lo, hi, str(device))
        f = self._freq_cache.get(key)
        if f is None:
            pos = joint_positions(h_tok, w_tok, text_len)[lo:hi]
            f = rope_freqs(pos, self.cfg.axes_dims, self.cfg.rope_theta).to(device)
            self._freq_cache[key] = f
        return f

    # -- forward ------------------------------------------------------------
    def forward_local(self, x_img: torch.Tensor, text: torch.Tensor, t: torch.Tensor, h_tok: int, w_tok: int,
                      sp: SPContext) -> Tuple[torch.Tensor, int, int]:
        """x_img: [B, N_img, patch_dim] patch features of all image tokens;
        text: [B, L, text_dim].  Returns the prediction for the image tokens in
        this rank's position range ([B, n_local_img, patch_dim]) and that range."""
        B, N, _ = x_img.shape
        L = text.shape[1]
        lo, hi = self.local_range(N + L, sp)
        parts = []
        img_lo, img_hi = min(lo, N), min(hi, N)
        if img_hi > img_lo:
            xi = x_img[:, img_lo:img_hi]
            parts.append(LinearFunction.apply(xi, self.x_embedder.weight, self.x_embedder.bias))
        txt_lo, txt_hi = max(lo, N) - N, max(hi, N) - N
        if txt_hi > txt_lo:
            parts.append(LinearFunction.apply(text[:, txt_lo:txt_hi], self.text_embedder.weight,
                                              self.text_embedder.bias))
        h = torch.cat(parts, 1) if len(parts) > 1 else parts[0]
        c = self.t_embedder(t * 1000.0)
        c_silu = SiLUFunction.apply(c)
        freqs = self.freqs_for(h_tok, w_tok, L, lo, hi, h.device)
        for blk in self.blocks:
            h = blk(h, c_silu, freqs, sp)
        out = self.final_layer(h, c_silu)
        return out[:, : img_hi - img_lo], img_lo, img_hi

    def forward(self, latent: torch.Tensor, text: torch.Tensor, t: torch.Tensor, sp: Optional[SPContext] = None):
        """Full-sequence convenience forward (single SP rank): returns the
        velocity prediction as a latent [B, C, H, W]."""
        sp = sp or SPContext.single()
        B, C, Hh, Ww = latent.shape
        p = self.cfg.patch_size
        x = self.patchify(latent)
        out, lo, hi = self.forward_local(x, text, t, Hh // p, Ww // p, sp)
        assert lo == 0 and hi == x.shape[1], "full forward needs sp=1; use forward_local for SP"
        return self.unpatchify(out, Hh, Ww)


def flow_matching_loss_local(model: DiT, latent: torch.Tensor, noise: torch.Tensor, text: torch.Tensor,
                             sigmas: torch.Tensor, sp: SPContext, weighting: Optional[torch.Tensor] = None):
    """Flow-matching MSE (train.py:454-501): x_t = (1-s) x0 + s eps, target = eps - x0
    (velocity; the reference's target is x0 - eps with the model predicting the
    negative velocity - the sign convention does not change the loss).
    Computed on this rank's image tokens and normalized by the global element
    count, so summing the per-rank losses gives the global mean."""
    B, C, Hh, Ww = latent.shape
    p = model.cfg.patch_size
    s = sigmas.view(B, 1, 1, 1).to(latent.dtype)
    x_t = (1.0 - s) * latent + s * noise
    target = noise - latent
    x = model.patchify(x_t)
    tgt = model.patchify(target)
    t = sigmas.float()
    pred, lo, hi = model.forward_local(x, text, t, Hh // p, Ww // p, sp)
    n_total = tgt.numel()
    if hi <= lo:
        return pred.float().sum() * 0.0
    diff = pred.float() - tgt[:, lo:hi].float()
    sq = diff.pow(2)
    if weighting is not None:
        sq = sq * weighting.view(B, 1, 1).float()
    return sq.sum() / n_total
