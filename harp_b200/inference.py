"""Sampling: classifier-free-guided Euler flow-matching inference for every
model family (reference: src/utils/inference.py:14-227, batch_image_inference).

Same steps as the reference's loop:
  * latents of shape [B, C, H/vae, W/vae] (or given initial latents);
  * mu from the image sequence length (calculate_shift), the scheduler's
    sigma grid with sigma_min forced to 0 (retrieve_timesteps);
  * per step, the model is run on [latents ; latents] with
    [positive ; negative] prompts when negative prompts are given; guidance
    pred = pos + g * (pos - neg), g = 0 once the normalised time passes
    cfg_truncation; optional renormalisation of pred to at most
    cfg_normalization x |pos|;
  * Euler update of the scheduler; decode with the VAE unless
    output_type == "latent".
Models are called through `velocity(model, latents, prompts, sigma)`, which
returns the noise - x0 velocity for DiT / MMDiT (trained on that target at
time sigma) and for the Z-Image layout (trained on x0 - noise at time 1 - sigma,
as the reference).  Inference runs on one SP rank (sp=1).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Union

import torch

from .parallel.sequence import SPContext
from .utils.diffusion import FlowMatchEulerDiscreteScheduler


def calculate_shift(image_seq_len: int, base_seq_len: int = 256, max_seq_len: int = 4096,
                    base_shift: float = 0.5, max_shift: float = 1.15) -> float:
    """mu grows linearly with the number of image tokens."""
    m = (max_shift - base_shift) / (max_seq_len - base_seq_len)
    return image_seq_len * m + (base_shift - m * base_seq_len)


def retrieve_timesteps(scheduler: FlowMatchEulerDiscreteScheduler, num_inference_steps: Optional[int] = None,
                       device=None, timesteps: Optional[Sequence[float]] = None,
                       sigmas: Optional[Sequence[float]] = None, **kwargs):
    if timesteps is not None and sigmas is not None:
        raise ValueError("pass at most one of timesteps / sigmas")
    scheduler.set_timesteps(num_inference_steps, device=device, timesteps=timesteps, sigmas=sigmas, **kwargs)
    return scheduler.timesteps, len(scheduler.timesteps)


def prepare_latents(batch_size, num_channels_latents, latent_height, latent_width, dtype, device, generator,
                    latents=None):
    shape = (batch_size, num_channels_latents, latent_height, latent_width)
    if latents is None:
        return torch.randn(shape, generator=generator, device="cpu" if generator is None or
                           generator.device.type == "cpu" else device, dtype=torch.float32).to(device, dtype)
    if tuple(latents.shape) != shape:
        raise ValueError(f"latents of shape {tuple(latents.shape)}, expected {shape}")
    return latents.to(device)


def _is_zimage(model) -> bool:
    return hasattr(model, "z_transformer")


@torch.no_grad()
def velocity(model, latents: torch.Tensor, prompts: List[torch.Tensor], sigma: torch.Tensor,
             metadata: Optional[torch.Tensor] = None, cond: Optional[List[torch.Tensor]] = None) -> torch.Tensor:
    """d x / d sigma predicted by `model` at noise level sigma [B] (noise - x0)."""
    sp = SPContext.single()
    if _is_zimage(model):
        imgs = list(latents.unsqueeze(2).unbind(0))
        out = model(x=imgs, t=1.0 - sigma, text_embedding=list(prompts), return_dict=False,
                    metadata=metadata, cond_list=cond, sp=sp)[0]
        return -torch.stack(out, 0).squeeze(2)
    text = torch.stack(list(prompts), 0) if isinstance(prompts, (list, tuple)) else prompts
    return model(latents, text, sigma.float(), sp)


@torch.no_grad()
def batch_image_inference(transformer, vae=None, scheduler: Optional[FlowMatchEulerDiscreteScheduler] = None,
                          image_processor=None, prompt_embeds: Sequence[torch.Tensor] = (),
                          negative_prompt_embeds: Optional[Sequence[torch.Tensor]] = None, height: int = 512,
                          width: int = 512, num_inference_steps: int = 50, sigmas: Optional[List[float]] = None,
                          guidance_scale: float = 5.0, cfg_normalization: Union[bool, float] = False,
                          cfg_truncation: float = 1.0, generator: Optional[torch.Generator] = None,
                          latents: Optional[torch.Tensor] = None, output_type: str = "latent",
                          return_dict: bool = True, joint_attention_kwargs: Optional[Dict[str, Any]] = None,
                          max_sequence_length: int = 512, initial_latents: Optional[torch.Tensor] = None,
                          vae_scale_factor: Optional[int] = None, in_channels: Optional[int] = None,
                          metadata: Optional[torch.Tensor] = None, cond: Optional[List[torch.Tensor]] = None,
                          progress: bool = False):
    scheduler = scheduler or FlowMatchEulerDiscreteScheduler()
    if vae_scale_factor is None:
        vae_scale_factor = 2 ** (len(vae.config.block_out_channels) - 1) if vae is not None else 8
    device = next(transformer.parameters()).device
    dtype = prompt_embeds[0].dtype
    B = len(prompt_embeds)
    if initial_latents is None:
        lh = 2 * (int(height) // (vae_scale_factor * 2))
        lw = 2 * (int(width) // (vae_scale_factor * 2))
        C = in_channels or getattr(transformer, "in_channels", None) or transformer.cfg.in_channels
        x = prepare_latents(B, C, lh, lw, dtype, device, generator, latents)
    else:
        x = initial_latents.to(device, dtype)
    seq = (x.shape[2] // 2) * (x.shape[3] // 2)
    cfg = scheduler.config
    mu = calculate_shift(seq, cfg.get("base_image_seq_len", 256), cfg.get("max_image_seq_len", 4096),
                         cfg.get("base_shift", 0.5), cfg.get("max_shift", 1.15))
    scheduler.sigma_min = 0.0
    timesteps, n = retrieve_timesteps(scheduler, num_inference_steps, device, sigmas=sigmas, mu=mu)
    use_cfg = negative_prompt_embeds is not None
    meta2 = torch.cat([metadata, metadata]) if (use_cfg and metadata is not None) else metadata
    cond2 = [torch.cat([c, c]) for c in cond] if (use_cfg and cond is not None) else cond
    it = range(n)
    if progress:
        from tqdm import tqdm

        it = tqdm(it)
    for i in it:
        sigma = scheduler.sigmas[i].to(device).expand(B)
        t_norm = 1.0 - float(scheduler.sigmas[i])  # normalised time: 0 at the start, 1 at the end
        if use_cfg:
            g = guidance_scale if t_norm <= cfg_truncation else 0.0
            v = velocity(transformer, torch.cat([x, x]), list(prompt_embeds) + list(negative_prompt_embeds),
                         torch.cat([sigma, sigma]), meta2, cond2).float()
            pos, neg = v[:B], v[B:]
            pred = pos + g * (pos - neg)
            if cfg_normalization:
                pn = torch.linalg.vector_norm(pos.flatten(1), dim=1)
                nn_ = torch.linalg.vector_norm(pred.flatten(1), dim=1)
                cap = pn * float(cfg_normalization)
                fac = torch.where(nn_ > cap, cap / nn_, torch.ones_like(nn_))
                pred = pred * fac.view(B, 1, 1, 1)
        else:
            pred = velocity(transformer, x, list(prompt_embeds), sigma, metadata, cond).float()
        x = scheduler.step(pred.to(dtype), timesteps[i], x, return_dict=False)[0].to(dtype)
    if output_type == "latent" or vae is None:
        image = x
    else:
        z = x / vae.config.scaling_factor + vae.config.shift_factor
        image = vae.decode(z.to(vae.dtype), return_dict=False)[0]
        if image_processor is not None:
            image = image_processor.postprocess(image, output_type=output_type)
    if not return_dict:
        return (image,)
    return {"images": image}
