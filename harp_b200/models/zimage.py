"""Z-Image DiT: the reference's model family, same module tree and state_dict
keys, running on the harp kernels.

Reference sources (layout and math):
  src/models/z_image/standalone_transformer.py
      RMSNorm :123-156, TimestepEmbedder :159-194, ZAttention :198-276,
      FeedForward :279-290, ZImageTransformerBlock :294-355, FinalLayer :358-372,
      RopeEmbedder :375-414, ZImageTransformer2DModel :417-755
  src/models/z_image/hl_model.py    Z_Transformer (SP wrapper, cond branch,
                                    metadata embedders) :37-453
  src/models/z_image/module/block.py, module/attn.py    Z_SingleBlock,
                                    Z_JointBlock, Z_Attention
State-dict layout of Z_Transformer (kept exactly):
  {noise_refiner,context_refiner,layers,cond_refiner_1,cond_refiner_2}.<i>.attention.attn.
      {to_q,to_k,to_v,to_out.0}.weight, {norm_q,norm_k}.weight
  ....z_block.{attention_norm1,attention_norm2,ffn_norm1,ffn_norm2}.weight,
      z_block.feed_forward.{w1,w2,w3}.weight, z_block.adaLN_modulation.0.{weight,bias}
  cond_embedder_{1,2}.{weight,bias}, cond_pad_token, meta_embeddings.<i>.mlp.{0,2}.*
  z_transformer.{all_x_embedder.2-1, all_final_layer.2-1.*, t_embedder.mlp.*,
      cap_embedder.{0,1}.*, x_pad_token, cap_pad_token}

Differences from the reference, on purpose:
  * residual math of the blocks follows the base model (x + gate*norm2(f(...)));
    HARP's block.py drops the MLP residual (block.py:44-49) - set
    `harp_block_compat=True` to reproduce that.
  * in the sequence-parallel wrapper, samples in a batch must have the same
    image size and caption length (the reference ignores attention masks in
    its ring attention too, attn.py:91-99); the base model's forward takes
    mixed sizes.
  * under sequence parallelism every embedder and the final layer run on the
    tokens a rank holds (never replicated), so summing parameter gradients
    over all ranks is exact; the reference instead replicates them and keeps
    only the owner's gradient (grad_manager.py:53-61).  There, the adaLN input
    passes through SPBroadcast (an all-reduce of its gradient) once per
    section (hl_model.py:174, 312, 439), so the sections' already summed
    gradients are summed again: with its own hl_model.py on two CPU ranks,
    the t_embedder and metadata-embedder gradients come out 1.97x the
    one-rank values.  The blocks' gradients agree with the one-rank run.
"""
from __future__ import annotations

import copy
import json
import math
import os
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from ..ops.modules import MySiLU, MyTanh, QKNormRopeFunction, kpLinear, kpRMSNorm, sp_attention
from ..parallel.sequence import SPContext

ADALN_EMBED_DIM = 256
SEQ_MULTI_OF = 32


def Linear(i, o, bias=True):
    return kpLinear(i, o, bias=bias, dtype=torch.float32)


def RMSNorm(dim, eps=1e-5):
    return kpRMSNorm(dim, eps=eps)


class TimestepEmbedder(nn.Module):
    def __init__(self, out_size, mid_size=None, frequency_embedding_size=256):
        super().__init__()
        mid_size = mid_size or out_size
        self.mlp = nn.Sequential(Linear(frequency_embedding_size, mid_size), nn.SiLU(), Linear(mid_size, out_size))
        self.frequency_embedding_size = frequency_embedding_size

    @staticmethod
    def timestep_embedding(t, dim, max_period=10000):
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        args = t[:, None].float() * freqs[None]
        emb = torch.cat([torch.cos(args), torch.sin(args)], -1)
        if dim % 2:
            emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], -1)
        return emb

    def forward(self, t):
        f = self.timestep_embedding(t, self.frequency_embedding_size).to(self.mlp[0].weight.dtype)
        h = self.mlp[0](f)
        h = MySiLU.apply(h)
        return self.mlp[2](h)


class ZAttention(nn.Module):
    def __init__(self, query_dim, heads, dim_head, qk_norm="rms_norm", eps=1e-5):
        super().__init__()
        inner = heads * dim_head
        self.heads, self.dim_head = heads, dim_head
        self.to_q = Linear(query_dim, inner, bias=False)
        self.to_k = Linear(query_dim, inner, bias=False)
        self.to_v = Linear(query_dim, inner, bias=False)
        self.to_out = nn.ModuleList([Linear(inner, query_dim, bias=False), nn.Identity()])
        self.norm_q = RMSNorm(dim_head, eps) if qk_norm else None
        self.norm_k = RMSNorm(dim_head, eps) if qk_norm else None

    def forward(self, x, freqs, sp: SPContext):
        """x [B, S, D]; freqs fp32 [B*S, Dh/2, 2] (per token row)."""
        H, Dh = self.heads, self.dim_head
        q, k, v = self.to_q(x), self.to_k(x), self.to_v(x)
        wq = self.norm_q.weight if self.norm_q is not None else None
        wk = self.norm_k.weight if self.norm_k is not None else None
        eps = self.norm_q.eps if self.norm_q is not None else 1e-5
        q, k = QKNormRopeFunction.apply(q, k, wq, wk, freqs, H, Dh, eps, self.norm_q is not None)
        o = sp_attention(q, k, v.contiguous(), H, Dh, sp)
        return self.to_out[0](o)


class FeedForward(nn.Module):
    def __init__(self, dim, hidden_dim):
        super().__init__()
        self.w1 = Linear(dim, hidden_dim, bias=False)
        self.w2 = Linear(hidden_dim, dim, bias=False)
        self.w3 = Linear(dim, hidden_dim, bias=False)

    def _forward_silu_gating(self, x1, x3):
        return MySiLU.apply(x1) * x3

    def forward(self, x):
        return self.w2(self._forward_silu_gating(self.w1(x), self.w3(x)))


class ZImageTransformerBlock(nn.Module):
    def __init__(self, layer_id, dim, n_heads, n_kv_heads, norm_eps, qk_norm, modulation=True):
        super().__init__()
        self.dim, self.layer_id = dim, layer_id
        self.head_dim = dim // n_heads
        self.attention = ZAttention(dim, n_heads, dim // n_heads, "rms_norm" if qk_norm else None, eps=1e-5)
        self.feed_forward = FeedForward(dim, int(dim / 3 * 8))
        self.attention_norm1 = RMSNorm(dim, norm_eps)
        self.ffn_norm1 = RMSNorm(dim, norm_eps)
        self.attention_norm2 = RMSNorm(dim, norm_eps)
        self.ffn_norm2 = RMSNorm(dim, norm_eps)
        self.modulation = modulation
        if modulation:
            self.adaLN_modulation = nn.Sequential(Linear(min(dim, ADALN_EMBED_DIM), 4 * dim, bias=True))

    def forward(self, x, freqs, adaln_input=None, sp: Optional[SPContext] = None, attention=None, compat=False):
        sp = sp or SPContext()
        attn = attention if attention is not None else self.attention
        if self.modulation:
            mod = self.adaLN_modulation(adaln_input).unsqueeze(1)
            scale_msa, gate_msa, scale_mlp, gate_mlp = mod.chunk(4, dim=2)
            gate_msa, gate_mlp = MyTanh.apply(gate_msa.contiguous()), MyTanh.apply(gate_mlp.contiguous())
            scale_msa, scale_mlp = 1.0 + scale_msa, 1.0 + scale_mlp
            a = attn(self.attention_norm1(x) * scale_msa, freqs, sp)
            x = x + gate_msa * self.attention_norm2(a)
            if compat:  # HARP block.py:44-49 (MLP residual dropped)
                h = self.feed_forward(self.ffn_norm1(x) * scale_mlp)
                return self.ffn_norm2(h) * gate_mlp + h
            return x + gate_mlp * self.ffn_norm2(self.feed_forward(self.ffn_norm1(x) * scale_mlp))
        a = attn(self.attention_norm1(x), freqs, sp)
        x = x + self.attention_norm2(a)
        if compat == "joint":  # HARP block.py:106-118: Z_JointBlock drops the input residual here too
            h = self.feed_forward(self.ffn_norm1(x))
            return h + self.ffn_norm2(h)
        # Z_SingleBlock keeps the base model's residual without modulation (block.py:51-58)
        return x + self.ffn_norm2(self.feed_forward(self.ffn_norm1(x)))


class FinalLayer(nn.Module):
    def __init__(self, hidden_size, out_channels):
        super().__init__()
        self.norm_final = nn.LayerNorm(hidden_size, elementwise_affine=False, eps=1e-6)
        self.linear = Linear(hidden_size, out_channels, bias=True)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), Linear(min(hidden_size, ADALN_EMBED_DIM), hidden_size))

    def forward(self, x, c):
        scale = 1.0 + self.adaLN_modulation[1](MySiLU.apply(c.contiguous()))
        y = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), eps=1e-6).to(x.dtype) * scale.unsqueeze(1)
        return self.linear(y)


class RopeEmbedder:
    """3-axis rotary tables: axis a of head_dim slice axes_dims[a] uses
    frequencies theta^(-2i/d_a) at integer positions; returns fp32 (cos, sin).
    The angle is formed in fp64 and rounded to fp32 before its cosine and sine,
    as the reference's precomputed tables are (standalone_transformer.py:388-398),
    so the rotations agree with a model trained there to fp32 rounding."""

    def __init__(self, theta=256.0, axes_dims=(16, 56, 56), axes_lens=(64, 128, 128)):
        self.theta, self.axes_dims, self.axes_lens = theta, tuple(axes_dims), tuple(axes_lens)

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        parts = []
        for a, d in enumerate(self.axes_dims):
            inv = 1.0 / (self.theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d))
            parts.append((ids[:, a].double()[:, None] * inv[None]).float())
        ang = torch.cat(parts, -1)
        return torch.stack([ang.cos(), ang.sin()], -1)

    def complex(self, ids):
        f = self(ids)
        return torch.complex(f[..., 0], f[..., 1])


class RopeTableEmbedder(RopeEmbedder):
    """RopeEmbedder that computes each axis's (cos, sin) table once per device
    (axes_lens[a] positions) and then only gathers rows by id, as the
    reference's table-lookup embedder does (kp_rope_embedder.py:46-67).  Same
    values as RopeEmbedder for ids inside the tables."""

    def __init__(self, theta=256.0, axes_dims=(16, 56, 56), axes_lens=(64, 128, 128)):
        super().__init__(theta, axes_dims, axes_lens)
        self._tables: Dict[torch.device, List[torch.Tensor]] = {}

    def tables(self, device) -> List[torch.Tensor]:
        device = torch.device(device)
        if device not in self._tables:
            tabs = []
            for a, (d, n) in enumerate(zip(self.axes_dims, self.axes_lens)):
                ids = torch.zeros(n, len(self.axes_dims), dtype=torch.int64, device=device)
                ids[:, a] = torch.arange(n, device=device)
                full = RopeEmbedder.__call__(self, ids)
                lo = sum(self.axes_dims[:a]) // 2
                tabs.append(full[:, lo:lo + d // 2].contiguous())
            self._tables[device] = tabs
        return self._tables[device]

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        tabs = self.tables(ids.device)
        return torch.cat([t[ids[:, a].long()] for a, t in enumerate(tabs)], 1)


# the reference's names (kp_rope_embedder.py:6, 46)
RopeEmbedderReference = RopeEmbedder
RopeEmbedderSVE = RopeTableEmbedder


def replace_ropeembedder_with_sverope(model: nn.Module, rope_class=RopeTableEmbedder) -> nn.Module:
    """Swap every `rope_embedder` attribute in the module tree for a
    `rope_class` with the same theta and axes (kp_rope_embedder.py:70-84)."""
    for mod in model.modules():
        emb = getattr(mod, "rope_embedder", None)
        if emb is not None and not isinstance(emb, rope_class):
            mod.rope_embedder = rope_class(theta=emb.theta, axes_dims=emb.axes_dims, axes_lens=emb.axes_lens)
    return model


class ConfigMixin:
    config_name = "config.json"

    @classmethod
    def load_config(cls, path, subfolder=None, revision=None):
        p = os.path.expanduser(path)
        if subfolder:
            p = os.path.join(p, subfolder)
        if os.path.isdir(p):
            p = os.path.join(p, cls.config_name)
        with open(p) as fh:
            return json.load(fh)

    @classmethod
    def from_config(cls, config):
        import inspect

        keys = set(inspect.signature(cls.__init__).parameters) - {"self"}
        return cls(**{k: v for k, v in dict(config).items() if k in keys})

    def save_config(self, directory):
        os.makedirs(directory, exist_ok=True)
        with open(os.path.join(directory, self.config_name), "w") as fh:
            json.dump(dict(self.config), fh, indent=2, sort_keys=True)


def _grid(size, start, device):
    axes = [torch.arange(s0, s0 + n, dtype=torch.int32, device=device) for s0, n in zip(start, size)]
    return torch.stack(torch.meshgrid(axes, indexing="ij"), -1)


def _pad_len(n: int) -> int:
    return (-n) % SEQ_MULTI_OF


class Z_Mixin:
    """Token layout of the legacy model (base.py:7-203): per sample, padded
    caption and image token runs, their position ids and pad masks, and one
    optional condition image."""

    @staticmethod
    def create_coordinate_grid(size, start=None, device=None) -> torch.Tensor:
        """int32 [*size, len(size)] grid of coordinates start[a] .. start[a] + size[a] - 1."""
        start = tuple(start) if start is not None else (0,) * len(size)
        axes = [torch.arange(s0, s0 + n, dtype=torch.int32, device=device) for s0, n in zip(start, size)]
        return torch.stack(torch.meshgrid(axes, indexing="ij"), -1)

    def unpatchify(self, x: List[torch.Tensor], size: List[Tuple], patch_size, f_patch_size,
                   out_channels) -> List[torch.Tensor]:
        """Token rows (padding at the end ignored) back to [C, F, H, W] per sample."""
        p, pf = patch_size, f_patch_size
        out = []
        for xi, (F_, H, W) in zip(x, size):
            n = (F_ // pf) * (H // p) * (W // p)
            out.append(xi[:n].view(F_ // pf, H // p, W // p, pf, p, p, out_channels)
                       .permute(6, 0, 3, 1, 4, 2, 5).reshape(out_channels, F_, H, W))
        return out

    def _pad_run(self, tokens: torch.Tensor, ids: torch.Tensor):
        """Pad a token run to a multiple of 32 by repeating its last row; pad
        ids are (0, 0, 0).  Returns (tokens, pad_mask, ids)."""
        n = tokens.shape[0]
        k = _pad_len(n)
        dev = tokens.device
        mask = torch.zeros(n + k, dtype=torch.bool, device=dev)
        if k:
            mask[n:] = True
            tokens = torch.cat([tokens, tokens[-1:].expand(k, tokens.shape[1])], 0)
            ids = torch.cat([ids, torch.zeros(k, ids.shape[1], dtype=ids.dtype, device=dev)], 0)
        return tokens, mask, ids

    def cond_patchify_and_embed(self, cond: torch.Tensor, patch_size: int, start: int, device):
        """cond [C, H, W] -> (tokens [(n+pad), p*p*C], pad_mask, ids) with ids on
        the plane (start, h, w)."""
        p = patch_size
        C, H, W = cond.shape
        toks = cond.view(C, H // p, p, W // p, p).permute(1, 3, 2, 4, 0).reshape((H // p) * (W // p), p * p * C)
        ids = self.create_coordinate_grid((1, H // p, W // p), (start, 0, 0), device).flatten(0, 2)
        return self._pad_run(toks, ids)

    def patchify_and_embed(self, all_image: List[torch.Tensor], all_cap_feats: List[torch.Tensor], patch_size: int,
                           f_patch_size: int, cond_list: Optional[List[torch.Tensor]]):
        """Per sample: padded caption and image token runs with their position
        ids and pad masks (base.py:85-203).  Returns (images, captions,
        image_sizes, image_ids, caption_ids, image_pad_masks, caption_pad_masks,
        cond_out) where cond_out is None or (tokens, pad_masks, ids) lists."""
        p, pf = patch_size, f_patch_size
        dev = all_image[0].device
        imgs, caps, sizes, img_ids, cap_ids, img_masks, cap_masks = [], [], [], [], [], [], []
        cond_out = ([], [], []) if cond_list is not None else None
        for i, (image, cap) in enumerate(zip(all_image, all_cap_feats)):
            L = cap.shape[0]
            Lp = L + _pad_len(L)
            c_ids = self.create_coordinate_grid((Lp, 1, 1), (1, 0, 0), dev).flatten(0, 2)
            c_tok = torch.cat([cap, cap[-1:].expand(Lp - L, cap.shape[1])], 0) if Lp > L else cap
            c_mask = torch.arange(Lp, device=dev) >= L
            caps.append(c_tok), cap_ids.append(c_ids), cap_masks.append(c_mask)
            C, F_, H, W = image.shape
            sizes.append((F_, H, W))
            t = image.view(C, F_ // pf, pf, H // p, p, W // p, p).permute(1, 3, 5, 2, 4, 6, 0)
            toks = t.reshape((F_ // pf) * (H // p) * (W // p), pf * p * p * C)
            ids = self.create_coordinate_grid((F_ // pf, H // p, W // p), (Lp + 1, 0, 0), dev).flatten(0, 2)
            toks, mask, ids = self._pad_run(toks, ids)
            imgs.append(toks), img_ids.append(ids), img_masks.append(mask)
            if cond_out is not None:
                ct, cm, ci = self.cond_patchify_and_embed(cond_list[i], p, Lp + 2, dev)
                cond_out[0].append(ct), cond_out[1].append(cm), cond_out[2].append(ci)
        return imgs, caps, sizes, img_ids, cap_ids, img_masks, cap_masks, cond_out


class Z_HLMixin(Z_Mixin):
    """Token layout of the sequence-parallel model (hl_base.py:7-212): as
    Z_Mixin, but cond_list holds one list of per-sample condition images per
    condition branch, and branch j's ids sit on the plane padded caption
    length + 2 + j.  The condition runs come back as a dict {"c_p", "c_p_m",
    "c_p_p_id"} of per-branch lists (tokens, pad masks, ids), with at least
    two branches as in the reference."""

    def patchify_and_embed(self, all_image: List[torch.Tensor], all_cap_feats: List[torch.Tensor], patch_size: int,
                           f_patch_size: int, cond_list: Optional[List[List[torch.Tensor]]]):
        out = Z_Mixin.patchify_and_embed(self, all_image, all_cap_feats, patch_size, f_patch_size, None)
        if cond_list is None:
            return out
        dev = all_image[0].device
        nb = max(2, len(cond_list))
        cond = {"c_p": [[] for _ in range(nb)], "c_p_m": [[] for _ in range(nb)], "c_p_p_id": [[] for _ in range(nb)]}
        for i, cap in enumerate(all_cap_feats):
            base = cap.shape[0] + _pad_len(cap.shape[0]) + 2
            for j, branch in enumerate(cond_list):
                tok, mask, ids = self.cond_patchify_and_embed(branch[i], patch_size, base + j, dev)
                cond["c_p"][j].append(tok), cond["c_p_m"][j].append(mask), cond["c_p_p_id"][j].append(ids)
        return out[:7] + (cond,)


class Z_LoraBranches:
    """Parameter-group helpers shared by both wrappers (hl_model.py:339-394,
    model.py:284-336): meta-embedding grad switch and the LoRA target names of
    each branch."""

    def switch_meta_embedding_grad(self, grad_stat: bool = True) -> int:
        n = 0
        if self.meta_embeddings is not None:
            for p in self.meta_embeddings.parameters():
                p.requires_grad_(grad_stat)
                n += p.numel()
        return n

    def get_branch_lora_modules(self, branch_name: str) -> List[str]:
        """Names of the LoRA target linears of every block of a branch.  The
        names resolve in this module tree (attention.attn.*); the reference
        lists attention.* and stops after the first block."""
        names: List[str] = []
        for i, block in enumerate(getattr(self, branch_name)):
            pre = f"{branch_name}.{i}"
            names += [f"{pre}.attention.attn.to_q", f"{pre}.attention.attn.to_k", f"{pre}.attention.attn.to_v",
                      f"{pre}.attention.attn.to_out.0", f"{pre}.z_block.feed_forward.w1",
                      f"{pre}.z_block.feed_forward.w2", f"{pre}.z_block.feed_forward.w3"]
            if block.z_block.modulation:
                names.append(f"{pre}.z_block.adaLN_modulation.0")
        return names

    def get_noise_lora_branch(self, patch_size: int = 2, f_patch_size: int = 1) -> List[str]:
        key = f"{patch_size}-{f_patch_size}"
        return self.get_branch_lora_modules("noise_refiner") + [
            f"z_transformer.all_x_embedder.{key}", f"z_transformer.all_final_layer.{key}.linear",
            f"z_transformer.all_final_layer.{key}.adaLN_modulation.1"]

    def get_context_lora_branch(self) -> List[str]:
        return ["z_transformer.cap_embedder.1"] + self.get_branch_lora_modules("context_refiner")

    def get_main_lora_branch(self) -> List[str]:
        return self.get_branch_lora_modules("layers") + ["z_transformer.t_embedder.mlp.0",
                                                         "z_transformer.t_embedder.mlp.2"]



class ModelMixin:
    """The reference's model conveniences (standalone_transformer.py:91-121):
    device / dtype properties, no-op xformers switches, and gradient
    checkpointing, which here is real: with it enabled every transformer
    block's activations are recomputed in the backward
    (torch.utils.checkpoint, non-reentrant) instead of being kept.  Under
    sequence parallelism the recomputation repeats the block's exchanges in
    the backward, in the same order on every rank."""

    gradient_checkpointing = False

    @property
    def device(self) -> torch.device:
        for t in list(self.parameters()) + list(self.buffers()):
            return t.device
        return torch.device("cpu")

    @property
    def dtype(self) -> torch.dtype:
        for t in list(self.parameters()) + list(self.buffers()):
            return t.dtype
        return torch.float32

    def enable_xformers_memory_efficient_attention(self, *args, **kwargs):
        return self

    def disable_xformers_memory_efficient_attention(self):
        return self

    def gradient_checkpointing_enable(self):
        self.gradient_checkpointing = True

    def gradient_checkpointing_disable(self):
        self.gradient_checkpointing = False

    def _run_block(self, block, *args):
        if self.gradient_checkpointing and torch.is_grad_enabled():
            import torch.utils.checkpoint as ckpt

            return ckpt.checkpoint(block, *args, use_reentrant=False)
        return block(*args)


class ZImageTransformer2DModel(nn.Module, ModelMixin, ConfigMixin):
    def __init__(self, all_patch_size=(2,), all_f_patch_size=(1,), in_channels=16, dim=3840, n_layers=30,
                 n_refiner_layers=2, n_heads=30, n_kv_heads=30, norm_eps=1e-5, qk_norm=True, cap_feat_dim=2560,
                 rope_theta=256.0, t_scale=1000.0, axes_dims=(32, 48, 48), axes_lens=(1024, 512, 512)):
        super().__init__()
        self.in_channels = self.out_channels = in_channels
        self.all_patch_size, self.all_f_patch_size = tuple(all_patch_size), tuple(all_f_patch_size)
        self.dim, self.n_heads, self.t_scale = dim, n_heads, t_scale
        self.config = dict(all_patch_size=list(all_patch_size), all_f_patch_size=list(all_f_patch_size),
                           in_channels=in_channels, dim=dim, n_layers=n_layers, n_refiner_layers=n_refiner_layers,
                           n_heads=n_heads, n_kv_heads=n_kv_heads, norm_eps=norm_eps, qk_norm=qk_norm,
                           cap_feat_dim=cap_feat_dim, rope_theta=rope_theta, t_scale=t_scale,
                           axes_dims=list(axes_dims), axes_lens=list(axes_lens))
        xe, fl = {}, {}
        for p, f in zip(self.all_patch_size, self.all_f_patch_size):
            xe[f"{p}-{f}"] = Linear(f * p * p * in_channels, dim, bias=True)
            fl[f"{p}-{f}"] = FinalLayer(dim, p * p * f * in_channels)
        self.all_x_embedder = nn.ModuleDict(xe)
        self.all_final_layer = nn.ModuleDict(fl)
        self.noise_refiner = nn.ModuleList([ZImageTransformerBlock(1000 + i, dim, n_heads, n_kv_heads, norm_eps,
                                                                   qk_norm, True) for i in range(n_refiner_layers)])
        self.context_refiner = nn.ModuleList([ZImageTransformerBlock(i, dim, n_heads, n_kv_heads, norm_eps, qk_norm,
                                                                     False) for i in range(n_refiner_layers)])
        self.t_embedder = TimestepEmbedder(min(dim, ADALN_EMBED_DIM), mid_size=1024)
        self.cap_embedder = nn.Sequential(RMSNorm(cap_feat_dim, norm_eps), Linear(cap_feat_dim, dim, bias=True))
        self.x_pad_token = nn.Parameter(torch.zeros(1, dim))
        self.cap_pad_token = nn.Parameter(torch.zeros(1, dim))
        self.layers = nn.ModuleList([ZImageTransformerBlock(i, dim, n_heads, n_kv_heads, norm_eps, qk_norm)
                                     for i in range(n_layers)])
        assert dim // n_heads == sum(axes_dims)
        self.rope_embedder = RopeEmbedder(rope_theta, axes_dims, axes_lens)

    # -- token layout helpers (standalone_transformer.py:533-644): patchify without padding (the SP
    #    wrapper pads its runs itself), unpatchify of one sample, position ids --
    def patchify(self, images: List[torch.Tensor], patch_size: int, f_patch_size: int):
        out, sizes = [], []
        for img in images:
            C, F_, H, W = img.shape
            pF, pH, pW = f_patch_size, patch_size, patch_size
            sizes.append((F_, H, W))
            t = img.view(C, F_ // pF, pF, H // pH, pH, W // pW, pW).permute(1, 3, 5, 2, 4, 6, 0)
            out.append(t.reshape((F_ // pF) * (H // pH) * (W // pW), pF * pH * pW * C))
        return out, sizes

    def unpatchify(self, x: torch.Tensor, size, patch_size, f_patch_size):
        F_, H, W = size
        pF, pH = f_patch_size, patch_size
        n = (F_ // pF) * (H // pH) * (W // pH)
        return (x[:n].view(F_ // pF, H // pH, W // pH, pF, pH, pH, self.out_channels)
                .permute(6, 0, 3, 1, 4, 2, 5).reshape(self.out_channels, F_, H, W))

    def positions(self, cap_len: int, grid: Tuple[int, int, int], device) -> Tuple[torch.Tensor, torch.Tensor]:
        cap_pad = (-cap_len) % SEQ_MULTI_OF
        cap_ids = _grid((cap_len + cap_pad, 1, 1), (1, 0, 0), device).flatten(0, 2)
        img_ids = _grid(grid, (cap_len + cap_pad + 1, 0, 0), device).flatten(0, 2)
        return img_ids, cap_ids

    def forward(self, x: List[torch.Tensor], t, cap_feats: List[torch.Tensor], patch_size=2, f_patch_size=1,
                return_dict=True, sp: Optional[SPContext] = None):
        """Single-rank forward (standalone_transformer.py:557-755) on samples of
        any image size and caption length.

        As in the reference, each sample's image and caption token runs are
        padded to a multiple of 32 (SEQ_MULTI_OF) with the learned pad tokens at
        position id (0, 0, 0), and the pad tokens are attended to; only the
        padding that batches samples of different lengths is masked there.
        Here samples with the same image size and caption length run together
        as one dense batch instead, so no mask is needed and the attention
        sees real rows only: the same result for every real token."""
        sp = sp or SPContext()
        key = f"{patch_size}-{f_patch_size}"
        c = self.t_embedder(t * self.t_scale)
        imgs, caps, sizes, img_ids, cap_ids, _, _, _ = Z_Mixin().patchify_and_embed(x, cap_feats, patch_size,
                                                                                   f_patch_size, None)
        groups: Dict[tuple, List[int]] = {}
        for i in range(len(x)):
            groups.setdefault((sizes[i], cap_feats[i].shape[0]), []).append(i)
        res: List[Optional[torch.Tensor]] = [None] * len(x)
        for ((F_, H, W), L), idx in groups.items():
            n = len(idx)
            xs = self.all_x_embedder[key](torch.stack([imgs[i] for i in idx]))
            adaln = c.index_select(0, torch.tensor(idx, device=c.device)).to(xs.dtype)
            n_img = (F_ // f_patch_size) * (H // patch_size) * (W // patch_size)
            if xs.shape[1] > n_img:
                pad = self.x_pad_token.to(xs.dtype).expand(n, xs.shape[1] - n_img, -1)
                xs = torch.cat([xs[:, :n_img], pad], 1)
            cs = self.cap_embedder(torch.stack([caps[i] for i in idx]).to(xs.dtype))
            if cs.shape[1] > L:
                pad = self.cap_pad_token.to(cs.dtype).expand(n, cs.shape[1] - L, -1)
                cs = torch.cat([cs[:, :L], pad], 1)
            f_img = self.rope_embedder(img_ids[idx[0]])
            f_cap = self.rope_embedder(cap_ids[idx[0]])
            rep_img = f_img.repeat(n, 1, 1)
            for layer in self.noise_refiner:
                xs = self._run_block(layer, xs, rep_img, adaln, sp)
            rep_cap = f_cap.repeat(n, 1, 1)
            for layer in self.context_refiner:
                cs = self._run_block(layer, cs, rep_cap)
            uni = torch.cat([xs, cs], 1)
            f_uni = torch.cat([f_img, f_cap], 0).repeat(n, 1, 1)
            for layer in self.layers:
                uni = self._run_block(layer, uni, f_uni, adaln, sp)
            out = self.all_final_layer[key](uni, adaln)
            for j, i in enumerate(idx):
                res[i] = self.unpatchify(out[j], sizes[i], patch_size, f_patch_size)
        return (res,) if not return_dict else {"sample": res}


# ---------------------------------------------------------------------------
# HARP SP wrapper (hl_model.py) with its block/attention wrappers
# ---------------------------------------------------------------------------
class Z_Attention(nn.Module):
    """module/attn.py:51-105: holds the pretrained ZAttention as `attn`."""

    def __init__(self, pretrained_attn: ZAttention, sp_size: int = 1):
        super().__init__()
        self.attn = pretrained_attn
        self.sp_size = sp_size

    def forward(self, x, freqs, sp):
        return self.attn(x, freqs, sp)


class Z_SingleBlock(nn.Module):
    """module/block.py:10-60: the base block as `z_block`, its attention re-routed."""

    def __init__(self, pretrained_block: ZImageTransformerBlock, sp_size: int = 1, compat: bool = False):
        super().__init__()
        self.attention = Z_Attention(pretrained_block.attention, sp_size)
        pretrained_block.attention = None
        self.z_block = pretrained_block
        self.compat = compat

    def forward(self, hidden_states, attn_mask=None, RoPE_embeds=None, adaln_input=None, sp=None):
        return self.z_block(hidden_states, RoPE_embeds, adaln_input, sp, attention=self.attention, compat=self.compat)


class Z_JointBlock(Z_SingleBlock):
    """module/block.py:62-118: same as Z_SingleBlock except, with
    harp_block_compat and no modulation, the MLP output replaces the residual
    stream (h + norm2(h)) instead of being added to it."""

    def forward(self, hidden_states, attn_mask=None, RoPE_embeds=None, adaln_input=None, sp=None):
        return self.z_block(hidden_states, RoPE_embeds, adaln_input, sp, attention=self.attention,
                            compat="joint" if self.compat else False)


class Z_Transformer(nn.Module, ModelMixin, Z_HLMixin, Z_LoraBranches):
    """Sequence-parallel Z-Image with HARP's condition-image branch and metadata
    embedders (hl_model.py:37-109).  forward() takes the reference's arguments
    and returns its output (the full per-sample predictions on every rank);
    forward_local() returns this rank's image-token predictions and their
    range, the training path (zimage_loss_local)."""

    def __init__(self, z_transformer: ZImageTransformer2DModel, num_metadata: int = 0, in_channels=None,
                 use_cond: bool = False, sp_group_model=None, sp_size=None, cond_channels: int = 192,
                 harp_block_compat: bool = False):
        super().__init__()
        self.sp_group_model = sp_group_model
        self.out_channels = self.in_channels = in_channels or z_transformer.in_channels
        c = harp_block_compat
        if use_cond:
            self.cond_refiner_1 = nn.ModuleList([Z_SingleBlock(b, sp_size or 1, c)
                                                 for b in copy.deepcopy(z_transformer.noise_refiner)])
            self.cond_refiner_2 = nn.ModuleList([Z_SingleBlock(b, sp_size or 1, c)
                                                 for b in copy.deepcopy(z_transformer.noise_refiner)])
            self.cond_embedder_1 = Linear(2 * 2 * cond_channels, z_transformer.dim)
            self.cond_embedder_2 = Linear(2 * 2 * cond_channels, z_transformer.dim)
            self.cond_pad_token = nn.Parameter(z_transformer.x_pad_token.detach().clone())
        self.use_cond = use_cond
        self.noise_refiner = nn.ModuleList([Z_SingleBlock(b, sp_size or 1, c) for b in z_transformer.noise_refiner])
        z_transformer.noise_refiner = None
        self.context_refiner = nn.ModuleList([Z_SingleBlock(b, sp_size or 1, c)
                                              for b in z_transformer.context_refiner])
        z_transformer.context_refiner = None
        self.layers = nn.ModuleList([Z_JointBlock(b, sp_size or 1, c) for b in z_transformer.layers])
        z_transformer.layers = None
        self.z_transformer = z_transformer
        self.n_metadata = num_metadata
        self.meta_embeddings = (nn.ModuleList([TimestepEmbedder(min(z_transformer.dim, ADALN_EMBED_DIM),
                                                                mid_size=1024) for _ in range(num_metadata)])
                                if num_metadata > 0 else None)

    @property
    def config(self):
        return self.z_transformer.config

    def switch_cond_branch_grad(self, grad_stat: bool = True) -> int:
        """requires_grad of both condition branches (embedders and refiners);
        returns the number of parameters switched (0 without the branches)."""
        n = 0
        for j in (1, 2):
            for name in (f"cond_embedder_{j}", f"cond_refiner_{j}"):
                mod = getattr(self, name, None)
                if mod is not None:
                    for p in mod.parameters():
                        p.requires_grad_(grad_stat)
                        n += p.numel()
        return n

    def _cond_tokens(self, cond: torch.Tensor, patch_size: int):
        C, H, W = cond.shape
        t = cond.view(C, H // patch_size, patch_size, W // patch_size, patch_size).permute(1, 3, 2, 4, 0)
        return t.reshape((H // patch_size) * (W // patch_size), patch_size * patch_size * C)

    def forward_local(self, x: List[torch.Tensor], t, text_embedding: List[torch.Tensor], patch_size=2,
                      f_patch_size=1, metadata=None, cond_list=None, sp: Optional[SPContext] = None):
        """Returns (pred [B, n_local_img, p*p*C], img_lo, img_hi): this rank's
        predictions for the real image tokens img_lo..img_hi-1 (the training
        path: no gather of the predictions).

        As in the reference (hl_base.py:41-203, hl_model.py:114-330) the
        caption, image and condition-image token runs are each padded to a
        multiple of 32 (the last row repeated, then replaced by the learned pad
        token after embedding, position id (0, 0, 0)), and the pad tokens are
        part of the unified sequence that every layer attends over."""
        sp = sp or SPContext()
        zt = self.z_transformer
        B = len(x)
        dev = x[0].device
        c = zt.t_embedder(t * zt.t_scale)
        if metadata is not None and self.meta_embeddings is not None:
            for i, emb in enumerate(self.meta_embeddings):
                c = c + emb(metadata[:, i])
        imgs, sizes = zt.patchify(x, patch_size, f_patch_size)
        img = torch.stack(imgs)  # [B, N, pdim]
        cap = torch.stack(list(text_embedding))
        F_, H, W = sizes[0]
        grid = (F_ // f_patch_size, H // patch_size, W // patch_size)
        N, L = img.shape[1], cap.shape[1]
        img_ids, cap_ids = zt.positions(L, grid, dev)
        img, img_ids, N_pad = _pad_run(img, img_ids)
        L_pad = cap_ids.shape[0]
        if L_pad != L:
            cap = torch.cat([cap, cap[:, -1:].expand(B, L_pad - L, cap.shape[2])], 1)
        adaln = c.to(torch.bfloat16 if img.dtype == torch.bfloat16 else img.dtype)
        xs = _local(img, sp)
        xs = zt.all_x_embedder[f"{patch_size}-{f_patch_size}"](xs)
        lo_i, hi_i = _range(N_pad, sp)
        xs = _fill_pad(xs, lo_i, hi_i, N, N_pad, zt.x_pad_token)
        f_img = zt.rope_embedder(img_ids[lo_i:hi_i]).repeat(B, 1, 1)
        for layer in self.noise_refiner:
            xs = self._run_block(layer, xs, None, f_img, adaln, sp)
        caps = zt.cap_embedder(_local(cap, sp).to(xs.dtype))
        lo_c, hi_c = _range(L_pad, sp)
        f_cap = zt.rope_embedder(cap_ids[lo_c:hi_c]).repeat(B, 1, 1)
        caps = _fill_pad(caps, lo_c, hi_c, L, L_pad, zt.cap_pad_token)
        for layer in self.context_refiner:
            caps = self._run_block(layer, caps, None, f_cap, None, sp)
        streams = [(xs, N_pad), (caps, L_pad)]
        ids = [img_ids, cap_ids]
        if self.use_cond and cond_list is not None:
            for j, cl in enumerate(cond_list):
                ctoks = torch.stack([self._cond_tokens(cc, patch_size) for cc in cl])
                Nc = ctoks.shape[1]
                Hc, Wc = cl[0].shape[1:]
                cids = _grid((1, Hc // patch_size, Wc // patch_size), (L_pad + 2 + j, 0, 0), dev).flatten(0, 2)
                ctoks, cids, Nc_pad = _pad_run(ctoks, cids)
                emb = getattr(self, f"cond_embedder_{j + 1}")
                cs = emb(_local(ctoks.to(xs.dtype), sp))
                lo_k, hi_k = _range(Nc_pad, sp)
                cs = _fill_pad(cs, lo_k, hi_k, Nc, Nc_pad, self.cond_pad_token)
                f_c = zt.rope_embedder(cids[lo_k:hi_k]).repeat(B, 1, 1)
                for layer in getattr(self, f"cond_refiner_{j + 1}"):
                    cs = self._run_block(layer, cs, None, f_c, adaln, sp)
                streams.append((cs, Nc_pad))
                ids.append(cids)
        # unified sequence [img ; text ; cond...]: gather each stream, concatenate, take this rank's chunk
        full = [_gather_seq(s, sp) for s, _ in streams]
        uni_full = torch.cat(full, 1)
        uni = _local(uni_full, sp)
        all_ids = torch.cat(ids, 0)
        lo_u, hi_u = _range(all_ids.shape[0], sp)
        f_uni = zt.rope_embedder(all_ids[lo_u:hi_u]).repeat(B, 1, 1)
        for layer in self.layers:
            uni = self._run_block(layer, uni, None, f_uni, adaln, sp)
        out = zt.all_final_layer[f"{patch_size}-{f_patch_size}"](uni, adaln)
        img_lo, img_hi = min(lo_u, N), min(hi_u, N)
        self._chunk_len = hi_u - lo_u  # this rank's share of the unified sequence (read by forward)
        return out[:, : max(0, img_hi - img_lo)], img_lo, img_hi

    def forward(self, x, t, text_embedding, patch_size=2, f_patch_size=1, return_dict=True, metadata=None,
                cond_list=None, sp: Optional[SPContext] = None):
        """The reference's contract (hl_model.py:114-337): every rank gets the
        full predictions, one [C, F, H, W] per sample ({"sample": list}, or a
        1-tuple when return_dict is False).  Under sequence parallelism the
        ranks' image-token predictions are all-gathered; as in the reference,
        the gather's backward keeps this rank's part of the gradient, so a loss
        computed in full on every rank yields per-rank partial parameter
        gradients whose sum over the ranks is the gradient (harp's trainer
        sums them).  forward_local is the training path without the gather."""
        sp = sp or SPContext()
        pred, lo, hi = self.forward_local(x, t, text_embedding, patch_size, f_patch_size, metadata, cond_list, sp)
        C, F_, H, W = x[0].shape
        n_img = (F_ // f_patch_size) * (H // patch_size) * (W // patch_size)
        if sp.size > 1:
            from ..managers.shard_manager import SequenceAllGather

            c = self._chunk_len  # image tokens lead the unified sequence, so a rank's lie at its chunk's start
            pad = pred.new_zeros(pred.shape[0], c - pred.shape[1], pred.shape[2])
            pred = SequenceAllGather.apply(torch.cat([pred, pad], 1).contiguous(), sp.group)[:, :n_img]
        zt = self.z_transformer
        res = [zt.unpatchify(pred[b], tuple(x[b].shape[1:]), patch_size, f_patch_size) for b in range(len(x))]
        return {"sample": res} if return_dict else (res,)


def _pad_run(tok: torch.Tensor, ids: torch.Tensor):
    """Pad a [B, n, d] token run to a multiple of SEQ_MULTI_OF by repeating its
    last row, with position id (0, 0, 0) for the padding.  Returns (tokens,
    ids, padded length)."""
    n = tok.shape[1]
    k = (-n) % SEQ_MULTI_OF
    if k:
        tok = torch.cat([tok, tok[:, -1:].expand(tok.shape[0], k, tok.shape[2])], 1)
        ids = torch.cat([ids, ids.new_zeros(k, ids.shape[1])], 0)
    return tok, ids, n + k


def _fill_pad(x: torch.Tensor, lo: int, hi: int, n_real: int, n_pad: int, pad_token: torch.Tensor) -> torch.Tensor:
    """Replace the rows of positions >= n_real in the chunk lo..hi-1 of an
    embedded run (padded length n_pad) by the learned pad token.  Whenever the
    run has padding every rank uses the pad token, even with no pad row in its
    chunk (a zero gradient), so its gradient is reported on all ranks at the
    same point of the backward."""
    if n_real == n_pad:
        return x
    padm = torch.arange(lo, hi, device=x.device) >= n_real
    return torch.where(padm[None, :, None], pad_token.to(x.dtype), x)


def _range(n: int, sp: SPContext) -> Tuple[int, int]:
    assert n % sp.size == 0, f"sequence length {n} not divisible by sp={sp.size}"
    k = n // sp.size
    return sp.rank * k, (sp.rank + 1) * k


def _local(x: torch.Tensor, sp: SPContext) -> torch.Tensor:
    if sp.size == 1:
        return x
    lo, hi = _range(x.shape[1], sp)
    return x[:, lo:hi]


class _GatherSeq(torch.autograd.Function):
    """All-gather of a stream's chunks along dim 1 whose backward sums the
    gradient over the ranks before taking this rank's chunk.  After the
    gather every rank keeps a different chunk of the unified sequence (not a
    replicated copy), so a stream token's gradient can come from another rank;
    the reference's SequenceAllGather backward (own chunk only) assumes the
    replicated case."""

    @staticmethod
    def forward(ctx, x, group):
        from ..managers.shard_manager import _gather_dim1

        ctx.group = group
        return _gather_dim1(x, group)

    @staticmethod
    def backward(ctx, g):
        import torch.distributed as dist

        from ..managers.shard_manager import _chunk

        g = g.contiguous().clone()
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=ctx.group)
        return _chunk(g, ctx.group).contiguous(), None


def _gather_seq(x: torch.Tensor, sp: SPContext) -> torch.Tensor:
    if sp.size == 1:
        return x
    return _GatherSeq.apply(x.contiguous(), sp.group)


def zimage_loss_local(model: Z_Transformer, latent, noise, text, sigmas, sp: SPContext, metadata=None, cond=None,
                      weighting=None):
    """Flow-matching loss on this rank's image tokens, normalized by the global
    element count (summing over SP ranks gives the global mean)."""
    B = latent.shape[0]
    s = sigmas.view(B, 1, 1, 1).to(latent.dtype)
    x_t = (1.0 - s) * latent + s * noise
    target = latent - noise  # the reference's target (train.py:496)
    zt = model.z_transformer
    pred, lo, hi = model.forward_local(list(x_t.unsqueeze(2).unbind(0)), (1000 - sigmas * 1000) / 1000,
                                       list(text.unbind(0)), metadata=metadata, cond_list=cond, sp=sp)
    tgt, _ = zt.patchify(list(target.unsqueeze(2).unbind(0)), 2, 1)
    tgt = torch.stack(tgt)
    if hi <= lo:
        return pred.float().sum() * 0.0
    sq = (pred.float() - tgt[:, lo:hi].float()).pow(2)
    if weighting is not None:
        sq = sq * weighting.view(B, 1, 1).float()
    return sq.sum() / tgt.numel()


PRESETS = {
    "zimage-6b": dict(dim=3840, n_layers=30, n_refiner_layers=2, n_heads=30, cap_feat_dim=2560,
                      axes_dims=(32, 48, 48), axes_lens=(1024, 512, 512)),
    "zimage-tiny": dict(dim=256, n_layers=2, n_refiner_layers=1, n_heads=4, cap_feat_dim=64,
                        axes_dims=(16, 24, 24), axes_lens=(256, 64, 64)),
}
