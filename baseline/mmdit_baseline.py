"""Comparison baseline for the MMDiT / Flux configurations: a straightforward
torch.distributed NCCL + cuBLAS/SDPA implementation of the same
sequence-parallel training step.

Same model math as harp_b200.models.mmdit (double-stream blocks with separate
image/text weights meeting in one joint attention, single-stream parallel
blocks, adaLN modulation, RMSNorm, QK-RMSNorm, 3-axis RoPE, SwiGLU), built
from stock PyTorch pieces only:
  * linears: nn.functional.linear (cuBLAS)
  * attention: F.scaled_dot_product_attention over the K/V of every SP rank,
    gathered with the autograd-aware torch.distributed.nn all_gather (NCCL;
    its backward reduce-scatters dK/dV back to the owners)
  * replicated weights: DistributedDataParallel (NCCL all-reduce) with
    torch.optim.AdamW(fused=True) on fp32 master weights
  * sharded weights (shard=True): FSDP2 fully_shard per block (NCCL parameter
    all-gather before each block, gradient reduce-scatter after it), fp32
    sharded parameters and AdamW state, bf16 compute.  (offload=True would
    add FSDP2's pinned-host CPUOffloadPolicy; bench.py does not run it on
    B200: it raised an illegal memory access there.)
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
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from dit_baseline import joint_positions, rope_table  # noqa: E402


def apply_rope(x, freqs):  # x [B, S, H, D], freqs complex [S, D/2]; S may be 0
    B, S, H, Dh = x.shape
    xc = torch.view_as_complex(x.float().reshape(B, S, H, Dh // 2, 2))
    return torch.view_as_real(xc * freqs[None, :, None, :]).reshape(B, S, H, Dh).type_as(x)


def _cfg(name):
    # configuration numbers only (a dataclass of ints); no harp code runs on this path
    sys.path.insert(0, ROOT)
    from harp_b200.models.mmdit import PRESETS

    return PRESETS[name]


def _attend(q, k, v, sp_group, sp_size):
    """q, k, v [B, S_local, H, Dh]: attention of the local queries over every
    rank's keys (K/V all-gathered; the gather's backward reduce-scatters)."""
    if sp_size > 1:
        from torch.distributed.nn.functional import all_gather

        k = torch.cat(all_gather(k.contiguous(), group=sp_group), 1)
        v = torch.cat(all_gather(v.contiguous(), group=sp_group), 1)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return o.transpose(1, 2)


class Stream(nn.Module):
    def __init__(self, cfg, pre_only=False):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        self.pre_only = pre_only
        self.mod = nn.Linear(D, 2 * D if pre_only else 6 * D)
        self.qkv = nn.Linear(D, 3 * D)
        self.q_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        self.k_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        if not pre_only:
            self.proj = nn.Linear(D, D)
            self.w1 = nn.Linear(D, F_, bias=False)
            self.w3 = nn.Linear(D, F_, bias=False)
            self.w2 = nn.Linear(F_, D)

    def pre(self, x, c_silu, freqs, cfg):
        B, S, D = x.shape
        mod = self.mod(c_silu).unsqueeze(1)
        if self.pre_only:
            sh1, sc1 = mod.chunk(2, -1)
            rest = None
        else:
            sh1, sc1, g1, sh2, sc2, g2 = mod.chunk(6, -1)
            rest = (g1, sh2, sc2, g2)
        h = F.rms_norm(x, (D,), eps=cfg.norm_eps) * (1 + sc1) + sh1
        q, k, v = self.qkv(h).view(B, S, 3, cfg.heads, cfg.head_dim).unbind(2)
        return apply_rope(self.q_norm(q), freqs), apply_rope(self.k_norm(k), freqs), v, rest

    def post(self, x, o, rest, cfg):
        g1, sh2, sc2, g2 = rest
        x = x + g1 * self.proj(o)
        h = F.rms_norm(x, (x.shape[-1],), eps=cfg.norm_eps) * (1 + sc2) + sh2
        return x + g2 * self.w2(F.silu(self.w1(h)) * self.w3(h))


class DoubleBlock(nn.Module):
    def __init__(self, cfg, text_pre_only=False):
        super().__init__()
        self.cfg = cfg
        self.img = Stream(cfg)
        self.txt = Stream(cfg, pre_only=text_pre_only)

    def forward(self, x, n_img, c_silu, freqs, sp_group, sp_size):
        cfg = self.cfg
        B = x.shape[0]
        parts, qs, ks, vs = [], [], [], []
        # both streams run even when this rank holds none of a stream's tokens
        # (an empty slice), so every rank's gradients cover every parameter
        for st, xs, fs in ((self.img, x[:, :n_img], freqs[:n_img]), (self.txt, x[:, n_img:], freqs[n_img:])):
            q, k, v, rest = st.pre(xs, c_silu, fs, cfg)
            parts.append((st, xs, rest))
            qs.append(q), ks.append(k), vs.append(v)
        q, k, v = (torch.cat(t, 1) for t in (qs, ks, vs))
        o = _attend(q, k, v, sp_group, sp_size).reshape(B, -1, cfg.hidden)
        outs, off = [], 0
        for st, xs, rest in parts:
            n = xs.shape[1]
            outs.append(xs if st.pre_only else st.post(xs, o[:, off:off + n], rest, cfg))
            off += n
        return torch.cat(outs, 1)


class SingleBlock(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        D, F_ = cfg.hidden, cfg.ffn_hidden
        self.cfg = cfg
        self.mod = nn.Linear(D, 3 * D)
        self.linear1 = nn.Linear(D, 3 * D + 2 * F_)
        self.q_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        self.k_norm = nn.RMSNorm(cfg.head_dim, eps=1e-6)
        self.linear2 = nn.Linear(D + F_, D)

    def forward(self, x, n_img, c_silu, freqs, sp_group, sp_size):
        cfg = self.cfg
        B, S, D = x.shape
        F_ = cfg.ffn_hidden
        sh, sc, g = self.mod(c_silu).unsqueeze(1).chunk(3, -1)
        h = F.rms_norm(x, (D,), eps=cfg.norm_eps) * (1 + sc) + sh
        q, k, v, gg, uu = torch.split(self.linear1(h), [D, D, D, F_, F_], -1)
        shp = (B, S, cfg.heads, cfg.head_dim)
        q = apply_rope(self.q_norm(q.reshape(shp)), freqs)
        k = apply_rope(self.k_norm(k.reshape(shp)), freqs)
        o = _attend(q, k, v.reshape(shp), sp_group, sp_size).reshape(B, S, D)
        return x + g * self.linear2(torch.cat([o, F.silu(gg) * uu], -1))


class BaselineMMDiT(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        D = cfg.hidden
        self.cfg = cfg
        self.img_in = nn.Linear(cfg.patch_dim, D)
        self.txt_in = nn.Linear(cfg.text_dim, D)
        self.t1 = nn.Linear(256, D)
        self.t2 = nn.Linear(D, D)
        last = cfg.depth_double - 1
        self.double_blocks = nn.ModuleList([DoubleBlock(cfg, text_pre_only=(i == last and cfg.depth_single == 0))
                                            for i in range(cfg.depth_double)])
        self.single_blocks = nn.ModuleList([SingleBlock(cfg) for _ in range(cfg.depth_single)])
        self.final_ada = nn.Linear(D, 2 * D)
        self.final = nn.Linear(D, cfg.patch_dim)
        self._freqs = {}

    @torch.no_grad()
    def init_weights(self):
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.RMSNorm):
                nn.init.ones_(m.weight)
        for b in list(self.double_blocks) + list(self.single_blocks):
            for st in ((b.img, b.txt) if isinstance(b, DoubleBlock) else (b,)):
                nn.init.zeros_(st.mod.weight)
        nn.init.zeros_(self.final_ada.weight)

    def t_embed(self, t):
        half = 128
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        a = t[:, None].float() * freqs[None]
        e = torch.cat([a.cos(), a.sin()], -1).to(self.t1.weight.dtype)
        return self.t2(F.silu(self.t1(e)))

    def forward(self, x_img, text, t, h_tok, w_tok, sp_group, sp_size, sp_rank):
        B, N, _ = x_img.shape
        L = text.shape[1]
        n = (N + L) // sp_size
        lo, hi = sp_rank * n, (sp_rank + 1) * n
        il, ih = min(lo, N), min(hi, N)
        tl, th = max(lo, N) - N, max(hi, N) - N
        # both embedders run (on an empty slice where this rank holds no such token)
        h = torch.cat([self.img_in(x_img[:, il:ih]), self.txt_in(text[:, tl:th])], 1)
        c_silu = F.silu(self.t_embed(t * 1000.0))
        key = (h_tok, w_tok, L, lo, hi, str(h.device))
        if key not in self._freqs:
            pos = joint_positions(h_tok, w_tok, L)[lo:hi]
            self._freqs[key] = rope_table(pos, self.cfg.axes_dims, self.cfg.rope_theta).to(h.device)
        freqs = self._freqs[key]
        for blk in list(self.double_blocks) + list(self.single_blocks):
            h = blk(h, ih - il, c_silu, freqs, sp_group, sp_size)
        shift, scale = self.final_ada(c_silu).unsqueeze(1).chunk(2, -1)
        h = F.layer_norm(h, (h.shape[-1],), eps=1e-6) * (1 + scale) + shift
        return self.final(h)[:, : ih - il], il, ih


class BaselineMMDiTTrainer:
    """One training step per call: forward over this rank's tokens, backward,
    gradient sync, AdamW.  Every rank of the job is one SP group's member (sp =
    world) or a DP replica of an SP group (sp < world)."""

    def __init__(self, model_name, device, sp_size, depth=None, shard=False, offload=False):
        cfg = _cfg(model_name)
        if depth:
            cfg = replace(cfg, depth_double=min(cfg.depth_double, depth), depth_single=min(cfg.depth_single, depth))
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
        self.shard = shard and self.ws > 1
        if self.shard:
            from torch.distributed.fsdp import CPUOffloadPolicy, MixedPrecisionPolicy, fully_shard

            # the same fp32 initial weights as the replicated path, then sharded
            with torch.device("cpu" if offload else device):
                model = BaselineMMDiT(cfg)
            model.init_weights()
            mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
            kw = {"mp_policy": mp}
            if offload:
                kw["offload_policy"] = CPUOffloadPolicy(pin_memory=True)
            for blk in list(model.double_blocks) + list(model.single_blocks):
                fully_shard(blk, **kw)
            fully_shard(model, **kw)
            self.model = model
            self.params = list(model.parameters())
            self.opt = torch.optim.AdamW(self.params, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                         fused=not offload, foreach=offload or None)
            self.master = None
        else:
            model = BaselineMMDiT(cfg)
            model.init_weights()
            model = model.to(device=device, dtype=torch.bfloat16)
            self.master = [p.detach().float().clone() for p in model.parameters()]
            if self.ws > 1:
                model = nn.parallel.DistributedDataParallel(
                    model, device_ids=[device.index] if device.type == "cuda" else None, broadcast_buffers=False,
                    bucket_cap_mb=100, find_unused_parameters=False)
            self.model = model
            core = model.module if self.ws > 1 else model
            self.params = list(core.parameters())
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

        x, tgt = patchify(x_t), patchify(target)
        for q in self.params:
            q.grad = None
        pred, lo, hi = self.model(x, text, sigmas.float(), Hh // p, Ww // p, self.sp_group, self.sp_size,
                                  self.sp_rank)
        loss = (pred.float() - tgt[:, lo:hi].float()).pow(2).sum() / tgt.numel()
        loss.backward()
        if self.master is None:  # FSDP: fp32 sharded parameters, reduce-scattered gradients
            self.opt.step()
        else:
            for mp, q in zip(self.master, self.params):
                mp.grad = q.grad.float() if q.grad is not None else torch.zeros_like(mp)
            self.opt.step()
            with torch.no_grad():
                torch._foreach_copy_(self.params, self.master)
        l = loss.detach().reshape(1)
        if self.ws > 1:
            dist.all_reduce(l)
        return l

    def step(self, batch):
        d = self.device
        return float(self.train_step(batch["latent"].to(d, non_blocking=True), batch["noise"].to(d, non_blocking=True),
                                     batch["text"].to(d, non_blocking=True),
                                     batch["sigmas"].to(d, non_blocking=True)).item())
