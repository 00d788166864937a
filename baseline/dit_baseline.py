"""Comparison baseline: a straightforward torch.distributed NCCL + cuBLAS/SDPA
implementation of the same sequence-parallel DiT training step.

Same model math as harp_b200.models.dit (adaLN-zero, RMSNorm, 3-axis RoPE,
QK-RMSNorm, SwiGLU, joint attention over image+text tokens), built from stock
PyTorch pieces only:
  * linears: nn.functional.linear (cuBLAS)
  * attention: F.scaled_dot_product_attention over the K/V of every SP rank,
    gathered with the autograd-aware torch.distributed.nn all_gather (NCCL;
    its backward reduce-scatters dK/dV back to the owners)
  * gradients: DistributedDataParallel bucketed all-reduce (NCCL)
  * optimizer: torch.optim.AdamW(fused=True) on fp32 master weights
No harp kernel, model or engine code is used on this path.
"""
from __future__ import annotations

import math
import os
import sys
from dataclasses import replace

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(name):
    # configuration numbers only (a dataclass of ints); no harp code runs on this path
    sys.path.insert(0, ROOT)
    from harp_b200.models.dit import PRESETS

    return PRESETS[name]


def rope_table(pos, axes_dims, theta):
    parts = []
    for a, d in enumerate(axes_dims):
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
        parts.append(pos[:, a].double()[:, None] * inv[None, :])
    ang = torch.cat(parts, -1)
    return torch.polar(torch.ones_like(ang), ang).to(torch.complex64)


def joint_positions(h, w, L):
    hh, ww = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
    img = torch.stack([torch.full_like(hh, L + 1), hh, ww], -1).reshape(-1, 3)
    txt = torch.stack([torch.arange(1, L + 1), torch.zeros(L, dtype=torch.long), torch.zeros(L, dtype=torch.long)], -1)
    return torch.cat([img, txt], 0)


def apply_rope(x, freqs):  # x [B, S, H, D], freqs complex [S, D/2]
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * freqs[None, :, None, :]).flatten(3).type_as(x)


class Block(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        self.cfg = cfg
        self.ada = nn.Linear(D, 6 * D)
        self.qkv = nn.Linear(D, 3 * D)
        self.q_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        self.k_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        self.proj = nn.Linear(D, D)
        self.w1 = nn.Linear(D, F_, bias=False)
        self.w3 = nn.Linear(D, F_, bias=False)
        self.w2 = nn.Linear(F_, D)

    def forward(self, x, c_silu, freqs, sp_group, sp_size):
        cfg = self.cfg
        B, S, D = x.shape
        H, Dh = cfg.heads, cfg.head_dim
        sh1, sc1, g1, sh2, sc2, g2 = self.ada(c_silu).unsqueeze(1).chunk(6, -1)
        h = F.rms_norm(x, (D,), eps=cfg.norm_eps) * (1 + sc1) + sh1
        q, k, v = self.qkv(h).view(B, S, 3, H, Dh).unbind(2)
        q = apply_rope(self.q_norm(q), freqs)
        k = apply_rope(self.k_norm(k), freqs)
        if sp_size > 1:
            from torch.distributed.nn.functional import all_gather

            ks = all_gather(k.contiguous(), group=sp_group)
            vs = all_gather(v.contiguous(), group=sp_group)
            k = torch.cat(ks, 1)
            v = torch.cat(vs, 1)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        o = o.transpose(1, 2).reshape(B, S, D)
        x = x + g1 * self.proj(o)
        h = F.rms_norm(x, (D,), eps=cfg.norm_eps) * (1 + sc2) + sh2
        x = x + g2 * self.w2(F.silu(self.w1(h)) * self.w3(h))
        return x


class BaselineDiT(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        D = cfg.hidden
        self.cfg = cfg
        self.x_embedder = nn.Linear(cfg.patch_dim, D)
        self.text_embedder = nn.Linear(cfg.text_dim, D)
        self.t1 = nn.Linear(256, D)
        self.t2 = nn.Linear(D, D)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.depth)])
        self.final_ada = nn.Linear(D, 2 * D)
        self.final = nn.Linear(D, cfg.patch_dim)
        self._freqs = {}
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        for b in self.blocks:
            nn.init.zeros_(b.ada.weight)
        nn.init.zeros_(self.final_ada.weight)

    def t_embed(self, t):
        half = 128
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        a = t[:, None].float() * freqs[None]
        e = torch.cat([a.cos(), a.sin()], -1).to(self.t1.weight.dtype)
        return self.t2(F.silu(self.t1(e)))

    def forward_local(self, x_img, text, t, h_tok, w_tok, sp_group, sp_size, sp_rank):
        B, N, _ = x_img.shape
        L = text.shape[1]
        n = (N + L) // sp_size
        lo, hi = sp_rank * n, (sp_rank + 1) * n
        parts = []
        il, ih = min(lo, N), min(hi, N)
        if ih > il:
            parts.append(self.x_embedder(x_img[:, il:ih]))
        tl, th = max(lo, N) - N, max(hi, N) - N
        if th > tl:
            parts.append(self.text_embedder(text[:, tl:th]))
        h = torch.cat(parts, 1) if len(parts) > 1 else parts[0]
        c_silu = F.silu(self.t_embed(t * 1000.0))
        key = (h_tok, w_tok, L, lo, hi)
        if key not in self._freqs:
            pos = joint_positions(h_tok, w_tok, L)[lo:hi]
            self._freqs[key] = rope_table(pos, self.cfg.axes_dims, self.cfg.rope_theta).to(h.device)
        freqs = self._freqs[key]
        for blk in self.blocks:
            h = blk(h, c_silu, freqs, sp_group, sp_size)
        shift, scale = self.final_ada(c_silu).unsqueeze(1).chunk(2, -1)
        h = F.layer_norm(h, (h.shape[-1],), eps=1e-6) * (1 + scale) + shift
        out = self.final(h)
        return out[:, : ih - il], il, ih

    forward = forward_local


class BaselineTrainer:
    def __init__(self, model_name, device, sp_size, depth=None):
        cfg = _cfg(model_name)
        if depth:
            cfg = replace(cfg, depth=depth)
        self.cfg = cfg
        self.device = device
        self.ws = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.sp_size = sp_size
        self.sp_rank = self.rank % sp_size
        self.sp_group = None
        if self.ws > 1:
            for g in range(self.ws // sp_size):
                ranks = list(range(g * sp_size, (g + 1) * sp_size))
                pg = dist.new_group(ranks) if sp_size < self.ws else dist.group.WORLD
                if self.rank in ranks:
                    self.sp_group = pg
        torch.manual_seed(0)
        model = BaselineDiT(cfg).to(device=device, dtype=torch.bfloat16)
        self.master = [p.detach().float().clone().requires_grad_(False) for p in model.parameters()]
        if self.ws > 1:
            model = nn.parallel.DistributedDataParallel(model, device_ids=[device.index], broadcast_buffers=False,
                                                        bucket_cap_mb=100, find_unused_parameters=sp_size > 1)
        self.model = model
        self.core = model.module if self.ws > 1 else model
        self.opt = torch.optim.AdamW(self.master, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                     fused=True)

    def train_step(self, latent, noise, text, sigmas):
        B, C, Hh, Ww = latent.shape
        p = self.cfg.patch_size
        s = sigmas.view(B, 1, 1, 1).to(latent.dtype)
        x_t = (1 - s) * latent + s * noise
        target = noise - latent

        def patchify(z):
            return z.view(B, C, Hh // p, p, Ww // p, p).permute(0, 2, 4, 3, 5, 1).reshape(B, -1, p * p * C)

        x = patchify(x_t)
        tgt = patchify(target)
        m = self.model if self.ws > 1 else self.core
        fwd = m.module.forward_local if self.ws > 1 else m.forward_local
        if self.ws > 1:
            # route through DDP's forward so its reducer hooks are armed
            pred, lo, hi = m(x, text, sigmas.float(), Hh // p, Ww // p, self.sp_group, self.sp_size, self.sp_rank)
        else:
            pred, lo, hi = fwd(x, text, sigmas.float(), Hh // p, Ww // p, None, 1, 0)
        loss = (pred.float() - tgt[:, lo:hi].float()).pow(2).sum() / tgt.numel()
        for q in self.core.parameters():
            q.grad = None
        loss.backward()
        params = list(self.core.parameters())
        for mp, q in zip(self.master, params):
            mp.grad = q.grad.float() if q.grad is not None else torch.zeros_like(mp)
        self.opt.step()
        with torch.no_grad():
            torch._foreach_copy_(params, self.master)
        l = loss.detach().reshape(1)
        if self.ws > 1:
            dist.all_reduce(l)
        return l

    def step(self, batch):
        d = self.device
        return float(self.train_step(batch["latent"].to(d, non_blocking=True), batch["noise"].to(d, non_blocking=True),
                                     batch["text"].to(d, non_blocking=True),
                                     batch["sigmas"].to(d, non_blocking=True)).item())
