"""MMDiT / Flux-style DiT: double-stream joint blocks (+ single-stream blocks).

Presets: an SD3-style ~2.5B double-stream MMDiT and a ~12B Flux-like model
(19 double-stream + 38 single-stream blocks, hidden 3072, 24 heads x 128,
4096 image + 512 text tokens of dim 4096 in the benchmark configuration).  The
~2B joint-block benchmark model (hidden 2304, 24 blocks sharing weights between
image and text tokens) is the DiT family's "mmdit-2b" preset.  The reference has
only the Z-Image single-stream model; these families reuse the same op layer
(harp GEMM, RMSNorm, QK-norm+RoPE, sequence-parallel attention, SwiGLU).

Double-stream block: image and text tokens keep separate weights (adaLN
modulation, QKV, QK-norm, output projection, MLP) and meet in one joint
attention over [image ; text].  Single-stream block: one fused projection to
QKV and the MLP's gate/up, joint attention, one projection back from
[attention ; MLP] (the parallel-block formulation).

Sequence parallelism: the joint sequence [image ; text] is cut into `sp`
equal chunks; each rank applies the image weights to the image tokens of its
chunk and the text weights to its text tokens, so any SP size works.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn

from ..ops import functional as Fn
from ..ops.modules import LinearFunction, MySiLU, QKNormRopeFunction, RMSNormFunction, sp_attention
from ..parallel.sequence import SPContext
from .dit import FinalLayer, TimestepEmbedder, _Linear, joint_positions, rope_freqs


@dataclass
class MMDiTConfig:
    in_channels: int = 16
    patch_size: int = 2
    hidden: int = 2304
    heads: int = 18
    depth_double: int = 24
    depth_single: int = 0
    mlp_ratio: float = 4.0
    text_dim: int = 2304
    axes_dims: Tuple[int, int, int] = (16, 56, 56)
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @property
    def ffn_hidden(self):
        return int(self.hidden * self.mlp_ratio)

    @property
    def patch_dim(self):
        return self.patch_size * self.patch_size * self.in_channels


PRESETS = {
    # SD3-style double-stream MMDiT, ~2.5B: 24 joint blocks, hidden 1536, 24 heads x 64
    "sd3-2b": MMDiTConfig(hidden=1536, heads=24, depth_double=24, depth_single=0, text_dim=4096,
                          axes_dims=(16, 24, 24)),
    # Flux-like, ~11.8B: 19 double + 38 single blocks, hidden 3072, 24 heads x 128;
    # SwiGLU hidden 8/3 D has the parameter count of a GELU MLP of 4 D
    "flux-12b": MMDiTConfig(hidden=3072, heads=24, depth_double=19, depth_single=38, text_dim=4096,
                            mlp_ratio=8.0 / 3.0),
    # Lumina-like ~2.3B: 24 joint (single-stream) blocks over image + text tokens,
    # hidden 2304, 18 heads x 128, SwiGLU 8/3 D
    "mmdit-2b": MMDiTConfig(hidden=2304, heads=18, depth_double=0, depth_single=24, text_dim=2304,
                            mlp_ratio=8.0 / 3.0),
    "mmdit-tiny": MMDiTConfig(hidden=256, heads=2, depth_double=2, depth_single=0, text_dim=128,
                              axes_dims=(32, 48, 48)),
    "flux-tiny": MMDiTConfig(hidden=256, heads=2, depth_double=1, depth_single=2, text_dim=128,
                             axes_dims=(32, 48, 48)),
}


def _lin(x, m: _Linear):
    return LinearFunction.apply(x, m.weight, m.bias)


def _report_unused(module: nn.Module):
    """This rank holds none of the tokens `module` acts on in this step, so its
    parameters get no gradient: their (zeroed) gradient slots are complete now.
    Tells the trainer's overlapped gradient sync (a no-op without one), so the
    bucket that holds them is not left waiting for gradients that never come."""
    for p in module.parameters():
        cb = getattr(p, "_harp_grad_ready", None)
        if cb is not None:
            cb(p)


def _rms(x, eps, w=None):
    return RMSNormFunction.apply(x, w, eps)


class _QKNorm(nn.Module):
    def __init__(self, head_dim):
        super().__init__()
        self.query_norm = nn.Parameter(torch.ones(head_dim))
        self.key_norm = nn.Parameter(torch.ones(head_dim))


class _Stream(nn.Module):
    """Per-stream weights of a double-stream block.  A pre-only stream (the
    text stream of the last block when no single-stream block follows) only
    feeds keys/values to the joint attention: its output is never read, so it
    has no output projection or MLP."""

    def __init__(self, cfg: MMDiTConfig, pre_only: bool = False):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        self.pre_only = pre_only
        self.mod = nn.Sequential(nn.SiLU(), _Linear(D, 2 * D if pre_only else 6 * D))
        self.qkv = _Linear(D, 3 * D)
        self.norm = _QKNorm(cfg.head_dim)
        if pre_only:
            return
        self.proj = _Linear(D, D)
        w13 = torch.empty(2 * F_, D)
        self.w1 = _Linear(D, F_, bias=False, weight=w13[:F_])
        self.w3 = _Linear(D, F_, bias=False, weight=w13[F_:])
        self.w2 = _Linear(F_, D)

    def pre_attn(self, x, c_silu, freqs, cfg):
        mod = _lin(c_silu, self.mod[1]).unsqueeze(1)
        if self.pre_only:
            sh1, sc1 = mod.chunk(2, -1)
            rest = None
        else:
            sh1, sc1, g1, sh2, sc2, g2 = mod.chunk(6, -1)
            rest = (g1, sh2, sc2, g2)
        h = _rms(x, cfg.norm_eps) * (1 + sc1) + sh1
        q, k, v = _lin(h, self.qkv).chunk(3, -1)
        q, k = QKNormRopeFunction.apply(q.contiguous(), k.contiguous(), self.norm.query_norm, self.norm.key_norm,
                                        freqs, cfg.heads, cfg.head_dim, 1e-6, True)
        return q, k, v.contiguous(), rest

    def post_attn(self, x, o, mods, cfg):
        g1, sh2, sc2, g2 = mods
        x = x + g1 * _lin(o, self.proj)
        h = _rms(x, cfg.norm_eps) * (1 + sc2) + sh2
        m = MySiLU.apply(_lin(h, self.w1).contiguous()) * _lin(h, self.w3)
        return x + g2 * _lin(m, self.w2)


class DoubleStreamBlock(nn.Module):
    def __init__(self, cfg: MMDiTConfig, text_pre_only: bool = False):
        super().__init__()
        self.cfg = cfg
        self.img = _Stream(cfg)
        self.txt = _Stream(cfg, pre_only=text_pre_only)

    def forward(self, x, n_img, c_silu, freqs, sp):
        cfg = self.cfg
        B = x.shape[0]
        parts, qs, ks, vs, mods = [], [], [], [], []
        splits = [(self.img, x[:, :n_img], freqs[:n_img]), (self.txt, x[:, n_img:], freqs[n_img:])]
        for stream, xs, fs in splits:
            if xs.shape[1] == 0:
                _report_unused(stream)
                continue
            q, k, v, md = stream.pre_attn(xs, c_silu, fs.repeat(B, 1, 1), cfg)
            parts.append((stream, xs, md))
            qs.append(q), ks.append(k), vs.append(v)
        q, k, v = (torch.cat(t, 1) if len(t) > 1 else t[0] for t in (qs, ks, vs))
        o = sp_attention(q, k, v, cfg.heads, cfg.head_dim, sp)
        outs, off = [], 0
        for stream, xs, md in parts:
            n = xs.shape[1]
            outs.append(xs if stream.pre_only else stream.post_attn(xs, o[:, off:off + n], md, cfg))
            off += n
        return torch.cat(outs, 1) if len(outs) > 1 else outs[0]


class SingleStreamBlock(nn.Module):
    def __init__(self, cfg: MMDiTConfig):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        self.cfg = cfg
        self.mod = nn.Sequential(nn.SiLU(), _Linear(D, 3 * D))
        self.linear1 = _Linear(D, 3 * D + 2 * F_)
        self.norm = _QKNorm(cfg.head_dim)
        self.linear2 = _Linear(D + F_, D)

    def forward(self, x, n_img, c_silu, freqs, sp):
        cfg = self.cfg
        B = x.shape[0]
        D, F_ = cfg.hidden, cfg.ffn_hidden
        sh, sc, g = _lin(c_silu, self.mod[1]).unsqueeze(1).chunk(3, -1)
        h = _rms(x, cfg.norm_eps) * (1 + sc) + sh
        a = _lin(h, self.linear1)
        q, k, v, gg, uu = torch.split(a, [D, D, D, F_, F_], -1)
        q, k = QKNormRopeFunction.apply(q.contiguous(), k.contiguous(), self.norm.query_norm, self.norm.key_norm,
                                        freqs.repeat(B, 1, 1), cfg.heads, cfg.head_dim, 1e-6, True)
        o = sp_attention(q, k, v.contiguous(), cfg.heads, cfg.head_dim, sp)
        m = MySiLU.apply(gg.contiguous()) * uu
        return x + g * _lin(torch.cat([o, m], -1), self.linear2)


class MMDiT(nn.Module):
    def __init__(self, cfg: MMDiTConfig):
        super().__init__()
        self.cfg = cfg
        D = cfg.hidden
        self.img_in = _Linear(cfg.patch_dim, D)
        self.txt_in = _Linear(cfg.text_dim, D)
        self.time_in = TimestepEmbedder(D, mid_size=D)
        last = cfg.depth_double - 1
        self.double_blocks = nn.ModuleList([DoubleStreamBlock(cfg, text_pre_only=(i == last and cfg.depth_single == 0))
                                            for i in range(cfg.depth_double)])
        self.single_blocks = nn.ModuleList([SingleStreamBlock(cfg) for _ in range(cfg.depth_single)])
        self.final_layer = FinalLayer(D, cfg.patch_dim)
        self._freq_cache = {}

    @torch.no_grad()
    def initialize_weights(self, seed: int = 0):
        for i, (name, p) in enumerate(self.named_parameters()):
            if name.endswith("bias"):
                p.zero_()
            elif "norm" in name:
                p.fill_(1.0)
            elif ".mod." in name or "adaLN_modulation" in name:
                p.zero_()
            else:
                bound = math.sqrt(6.0 / (p.shape[0] + p.shape[1]))
                Fn.philox_uniform_(p.data, seed, i << 32, -bound, bound)
        Fn.philox_uniform_(self.final_layer.linear.weight.data, seed, 0xFFFF << 32, -1e-3, 1e-3)

    def forward_local(self, x_img, text, t, h_tok, w_tok, sp: SPContext):
        B, N, _ = x_img.shape
        L = text.shape[1]
        S = N + L
        assert S % sp.size == 0
        n = S // sp.size
        lo, hi = sp.rank * n, (sp.rank + 1) * n
        il, ih = min(lo, N), min(hi, N)
        tl, th = max(lo, N) - N, max(hi, N) - N
        parts = []
        if ih > il:
            parts.append(_lin(x_img[:, il:ih], self.img_in))
        else:
            _report_unused(self.img_in)
        if th > tl:
            parts.append(_lin(text[:, tl:th], self.txt_in))
        else:
            _report_unused(self.txt_in)
        h = torch.cat(parts, 1) if len(parts) > 1 else parts[0]
        c_silu = MySiLU.apply(self.time_in(t * 1000.0))
        key = (h_tok, w_tok, L, lo, hi, str(h.device))
        freqs = self._freq_cache.get(key)
        if freqs is None:
            freqs = rope_freqs(joint_positions(h_tok, w_tok, L)[lo:hi], self.cfg.axes_dims,
                               self.cfg.rope_theta).to(h.device)
            self._freq_cache[key] = freqs
        n_img = ih - il
        for blk in self.double_blocks:
            h = blk(h, n_img, c_silu, freqs, sp)
        for blk in self.single_blocks:
            h = blk(h, n_img, c_silu, freqs, sp)
        out = self.final_layer(h, c_silu)
        return out[:, :n_img], il, ih

    def patchify(self, latent):
        B, C, H, W = latent.shape
        p = self.cfg.patch_size
        return latent.view(B, C, H // p, p, W // p, p).permute(0, 2, 4, 3, 5, 1).reshape(B, -1, p * p * C)

    def unpatchify(self, x, H, W):
        B = x.shape[0]
        p, C = self.cfg.patch_size, self.cfg.in_channels
        return x.view(B, H // p, W // p, p, p, C).permute(0, 5, 1, 3, 2, 4).reshape(B, C, H, W)

    def forward(self, latent, text, t, sp: Optional[SPContext] = None):
        """Full-sequence forward (one SP rank): velocity prediction [B, C, H, W]."""
        sp = sp or SPContext.single()
        B, C, H, W = latent.shape
        p = self.cfg.patch_size
        out, lo, hi = self.forward_local(self.patchify(latent), text, t, H // p, W // p, sp)
        assert lo == 0 and hi == (H // p) * (W // p), "full forward needs sp=1"
        return self.unpatchify(out, H, W)


def mmdit_loss_local(model: MMDiT, latent, noise, text, sigmas, sp: SPContext, weighting=None, **_):
    B, C, H, W = latent.shape
    p = model.cfg.patch_size
    s = sigmas.view(B, 1, 1, 1).to(latent.dtype)
    x = model.patchify((1 - s) * latent + s * noise)
    tgt = model.patchify(noise - latent)
    pred, lo, hi = model.forward_local(x, text, sigmas.float(), H // p, W // p, sp)
    if hi <= lo:
        return pred.float().sum() * 0.0
    sq = (pred.float() - tgt[:, lo:hi].float()).pow(2)
    if weighting is not None:
        sq = sq * weighting.view(B, 1, 1).float()
    return sq.sum() / tgt.numel()
