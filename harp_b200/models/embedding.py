"""Timestep embeddings (reference: src/models/embedding.py:7-158).

  get_timestep_embedding(t, dim, flip_sin_to_cos, downscale_freq_shift, scale, max_period)
      sinusoidal embedding of the DDPM paper: frequencies
      max_period ** (-i / (half - downscale_freq_shift)), [sin | cos] (or
      [cos | sin] when flipped), zero column appended for odd dims
  Timesteps(num_channels, flip_sin_to_cos, downscale_freq_shift)   module form
  TimestepEmbedding(in_channels, time_embed_dim, act_fn, out_dim, post_act_fn, cond_proj_dim)
      linear_1 -> act -> linear_2 (-> post_act), optional cond_proj added first
  TimestepEmbedder(out_size, mid_size, frequency_embedding_size)
      [cos | sin] embedding (period 10000, frequencies over half) -> mlp.{0,2}

Parameter names match the reference's (they are part of the checkpoint
layout); the Linear layers run through the harp GEMM.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from ..ops.modules import LinearFunction, MySiLU

_ACTS = {"silu": nn.SiLU, "mish": nn.Mish, "gelu": nn.GELU}


def get_timestep_embedding(timesteps: torch.Tensor, embedding_dim: int, flip_sin_to_cos: bool = False,
                           downscale_freq_shift: float = 1, scale: float = 1, max_period: int = 10000) -> torch.Tensor:
    assert timesteps.dim() == 1, "timesteps must be a 1-D tensor"
    half = embedding_dim // 2
    k = torch.arange(half, dtype=torch.float32, device=timesteps.device)
    freqs = torch.exp(-math.log(max_period) * k / (half - downscale_freq_shift))
    arg = scale * (timesteps[:, None].float() * freqs[None, :])
    sin, cos = torch.sin(arg), torch.cos(arg)
    emb = torch.cat([cos, sin], -1) if flip_sin_to_cos else torch.cat([sin, cos], -1)
    if embedding_dim % 2 == 1:
        emb = torch.nn.functional.pad(emb, (0, 1))
    return emb


class Timesteps(nn.Module):
    def __init__(self, num_channels: int, flip_sin_to_cos: bool, downscale_freq_shift: float):
        super().__init__()
        self.num_channels, self.flip_sin_to_cos = num_channels, flip_sin_to_cos
        self.downscale_freq_shift = downscale_freq_shift

    def forward(self, timesteps: torch.Tensor) -> torch.Tensor:
        return get_timestep_embedding(timesteps, self.num_channels, flip_sin_to_cos=self.flip_sin_to_cos,
                                      downscale_freq_shift=self.downscale_freq_shift)


def _lin(m: nn.Linear, x: torch.Tensor) -> torch.Tensor:
    return LinearFunction.apply(x, m.weight, m.bias)


class TimestepEmbedding(nn.Module):
    def __init__(self, in_channels: int, time_embed_dim: int, act_fn: str = "silu", out_dim: Optional[int] = None,
                 post_act_fn: Optional[str] = None, cond_proj_dim: Optional[int] = None):
        super().__init__()
        if act_fn not in _ACTS or (post_act_fn is not None and post_act_fn not in _ACTS):
            raise ValueError(f"activation must be one of {sorted(_ACTS)}")
        self.linear_1 = nn.Linear(in_channels, time_embed_dim)
        self.cond_proj = nn.Linear(cond_proj_dim, in_channels, bias=False) if cond_proj_dim is not None else None
        self.act = _ACTS[act_fn]()
        self.linear_2 = nn.Linear(time_embed_dim, out_dim if out_dim is not None else time_embed_dim)
        self.post_act = _ACTS[post_act_fn]() if post_act_fn is not None else None

    def forward(self, sample: torch.Tensor, condition: Optional[torch.Tensor] = None) -> torch.Tensor:
        if condition is not None:
            sample = sample + _lin(self.cond_proj, condition)
        h = _lin(self.linear_1, sample)
        h = MySiLU.apply(h) if isinstance(self.act, nn.SiLU) else self.act(h)
        h = _lin(self.linear_2, h)
        if self.post_act is not None:
            h = self.post_act(h)
        return h


class TimestepEmbedder(nn.Module):
    def __init__(self, out_size: int, mid_size: Optional[int] = None, frequency_embedding_size: int = 256):
        super().__init__()
        mid_size = mid_size or out_size
        self.mlp = nn.Sequential(nn.Linear(frequency_embedding_size, mid_size, bias=True), nn.SiLU(),
                                 nn.Linear(mid_size, out_size, bias=True))
        self.frequency_embedding_size = frequency_embedding_size

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000) -> torch.Tensor:
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        arg = t[:, None].float() * freqs[None]
        emb = torch.cat([torch.cos(arg), torch.sin(arg)], -1)
        if dim % 2:
            emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], -1)
        return emb

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        f = self.timestep_embedding(t, self.frequency_embedding_size)
        if self.mlp[0].weight.dtype.is_floating_point:
            f = f.to(self.mlp[0].weight.dtype)
        h = MySiLU.apply(_lin(self.mlp[0], f))
        return _lin(self.mlp[2], h)
