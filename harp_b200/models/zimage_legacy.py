"""Non-sequence-parallel Z-Image wrapper with variable-size samples (the
reference's legacy model).

Reference: src/models/z_image/model.py:1-349 (Z_Transformer over a diffusers
ZImageTransformer2DModel) and src/models/z_image/base.py:1-203 (Z_Mixin:
patchify_and_embed, cond_patchify_and_embed, unpatchify,
create_coordinate_grid).  The reference trainer never imports it.

Semantics kept from the reference:
  * every caption, image and condition-image token run is padded to a multiple
    of 32 tokens (SEQ_MULTI_OF); padded caption/image/condition tokens become
    the learned pad tokens, take position id (0, 0, 0) and ARE attended to
    (the attention mask only hides the padding that batches samples of
    different lengths together);
  * image position ids start after the padded caption (axis 0 = caption
    length + padding + 1), condition-image ids one further (+ 2);
  * the unified sequence of a sample is [image ; caption ; condition].

Here, instead of padding the batch to its longest sample and masking the
attention, samples with the same padded token counts and image sizes are run
together as one dense batch (no masks: the attention kernel sees only real
rows), which gives the masked computation's result for every real token.
The base model is harp_b200.models.zimage.ZImageTransformer2DModel (same
state-dict keys as the diffusers class; diffusers is not needed).
"""
from __future__ import annotations

import copy
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from ..parallel.sequence import SPContext
from .zimage import (ADALN_EMBED_DIM, Linear, ModelMixin, TimestepEmbedder, Z_JointBlock, Z_LoraBranches,
                     Z_Mixin, Z_SingleBlock, ZImageTransformer2DModel)


class Z_Transformer(nn.Module, ModelMixin, Z_Mixin, Z_LoraBranches):
    """Legacy (non-SP) Z-Image wrapper: noise/context/condition refiners and the
    joint layers over variable-size samples (model.py:20-349).

    z_transformer: the base model; its refiners and layers move into this
    module (as in the reference).  use_cond adds one condition-image branch
    (a refiner copied from the noise refiner, a 2x2x192 -> dim embedder and a
    pad token)."""

    def __init__(self, z_transformer: ZImageTransformer2DModel, num_metadata: int = 0,
                 in_channels: Optional[int] = None, use_cond: bool = False, cond_channels: int = 192,
                 harp_block_compat: bool = False):
        super().__init__()
        self.in_channels = self.out_channels = in_channels or z_transformer.in_channels
        c = harp_block_compat
        self.cond_embedder = None
        if use_cond:
            self.cond_refiner = nn.ModuleList([Z_SingleBlock(b, 1, c)
                                               for b in copy.deepcopy(z_transformer.noise_refiner)])
            self.cond_embedder = Linear(2 * 2 * cond_channels, z_transformer.dim)
            self.cond_pad_token = nn.Parameter(z_transformer.x_pad_token.detach().clone())
        self.noise_refiner = nn.ModuleList([Z_SingleBlock(b, 1, c) for b in z_transformer.noise_refiner])
        z_transformer.noise_refiner = None
        self.context_refiner = nn.ModuleList([Z_SingleBlock(b, 1, c) for b in z_transformer.context_refiner])
        z_transformer.context_refiner = None
        self.layers = nn.ModuleList([Z_JointBlock(b, 1, c) for b in z_transformer.layers])
        z_transformer.layers = None
        self.z_transformer = z_transformer
        self.n_metadata = num_metadata
        self.meta_embeddings = (nn.ModuleList([TimestepEmbedder(min(z_transformer.dim, ADALN_EMBED_DIM),
                                                                mid_size=1024) for _ in range(num_metadata)])
                                if num_metadata > 0 else None)

    @property
    def config(self):
        return self.z_transformer.config

    # -- forward ---------------------------------------------------------------
    def forward(self, x: List[torch.Tensor], t, text_embedding: List[torch.Tensor], patch_size=2, f_patch_size=1,
                return_dict: bool = True, metadata: Optional[torch.Tensor] = None,
                cond_list: Optional[List[torch.Tensor]] = None):
        """x: B images [C, F, H, W] (sizes may differ); t [B]; text_embedding: B
        caption features [L_i, cap_feat_dim]; cond_list: B condition images
        [cond_channels, H, W] or None.  Returns {"sample": B predictions
        [C, F, H, W]} (or a 1-tuple when return_dict is False)."""
        zt = self.z_transformer
        B = len(x)
        key = f"{patch_size}-{f_patch_size}"
        c = zt.t_embedder(t * zt.t_scale)
        if metadata is not None and self.meta_embeddings is not None:
            for i, emb in enumerate(self.meta_embeddings):
                c = c + emb(metadata[:, i])
        use_cond = cond_list is not None and self.cond_embedder is not None
        (imgs, caps, sizes, img_ids, cap_ids, img_masks, cap_masks,
         cond_out) = self.patchify_and_embed(x, text_embedding, patch_size, f_patch_size,
                                             cond_list if use_cond else None)
        # samples that share every padded length, image size and caption
        # length + padding form one dense batch
        groups: Dict[tuple, List[int]] = {}
        for i in range(B):
            k = (imgs[i].shape[0], caps[i].shape[0], sizes[i],
                 cond_out[0][i].shape[0] if use_cond else 0)
            groups.setdefault(k, []).append(i)
        out: List[Optional[torch.Tensor]] = [None] * B
        sp = SPContext()
        for idx in groups.values():
            n = len(idx)
            ix = torch.tensor(idx, device=c.device)
            adaln = c.index_select(0, ix)
            emb_x = zt.all_x_embedder[key](torch.stack([imgs[i] for i in idx]))
            dt = emb_x.dtype
            adaln = adaln.to(dt)
            m = torch.stack([img_masks[i] for i in idx])[..., None]
            xs = torch.where(m, zt.x_pad_token.to(dt), emb_x)
            f_x = zt.rope_embedder(img_ids[idx[0]])
            for layer in self.noise_refiner:
                xs = self._run_block(layer, xs, None, f_x.repeat(n, 1, 1), adaln, sp)
            caps_b = zt.cap_embedder(torch.stack([caps[i] for i in idx]).to(dt))
            m = torch.stack([cap_masks[i] for i in idx])[..., None]
            caps_b = torch.where(m, zt.cap_pad_token.to(dt), caps_b)
            f_c = zt.rope_embedder(cap_ids[idx[0]])
            for layer in self.context_refiner:
                caps_b = self._run_block(layer, caps_b, None, f_c.repeat(n, 1, 1), None, sp)
            seqs, fr = [xs, caps_b], [f_x, f_c]
            if use_cond:
                cs = self.cond_embedder(torch.stack([cond_out[0][i] for i in idx]).to(dt))
                m = torch.stack([cond_out[1][i] for i in idx])[..., None]
                cs = torch.where(m, self.cond_pad_token.to(dt), cs)
                f_k = zt.rope_embedder(cond_out[2][idx[0]])
                for layer in self.cond_refiner:
                    cs = self._run_block(layer, cs, None, f_k.repeat(n, 1, 1), adaln, sp)
                seqs.append(cs)
                fr.append(f_k)
            uni = torch.cat(seqs, 1)
            f_u = torch.cat(fr, 0).repeat(n, 1, 1)
            for layer in self.layers:
                uni = self._run_block(layer, uni, None, f_u, adaln, sp)
            pred = zt.all_final_layer[key](uni, adaln)
            for j, i in enumerate(idx):
                out[i] = pred[j, : imgs[i].shape[0]]
        res = self.unpatchify(out, sizes, patch_size, f_patch_size, self.out_channels)
        return {"sample": res} if return_dict else (res,)

    # -- parameter-group helpers (model.py:284-349; the others in Z_LoraBranches) --
    def switch_cond_branch_grad(self, grad_stat: bool = True) -> int:
        n = 0
        if self.cond_embedder is not None:
            for mod in (self.cond_embedder, self.cond_refiner):
                for p in mod.parameters():
                    p.requires_grad_(grad_stat)
                    n += p.numel()
        return n
