"""Helpers around the model: geo-metadata normalisation, RoPE application on
[B, H, S, D] tensors, trainable-parameter save hooks, VAE encoding, prompt
encoding, and deterministic fast initialisation.

Reference counterparts (src/utils/*, train.py):
  MetaData                  metadata.py:3-50   (lon/lat/gsd/year scaled to [0, scale])
  apply_rotary_emb          rope.py:6-66       (real (cos, sin) or complex freqs)
  save_*_hook               hook.py:5-39       (safetensors of trainable params)
  encode_images, preserve_requires_grad        utils.py:4-14
  encode_prompt, load_z_image_text_processer   vectorize.py:7-66 (Qwen3 hidden_states[-2])
  FastInitMode              train.py:274-285   (uniform_ -> fixed-seed Philox so every
                                                rank draws identical initial weights)
"""
from __future__ import annotations

import os
from contextlib import contextmanager
from typing import List, Sequence, Tuple, Union

import torch
from torch.utils._python_dispatch import TorchDispatchMode


class MetaData:
    """Normalised (lon, lat, gsd, year) vectors and caption text for
    geo-referenced images.  lon in [-base_lon, 180], lat in [-base_lat, 90],
    gsd in metres per pixel up to max_gsd, year up to 2100; each maps to
    [0, scale].  unnormalize(is_print=True) shifts lon / lat back by the base
    and the year by base_year (0 by default; the reference reads an unset
    attribute there)."""

    def __init__(self, base_lon: float = 180, base_lat: float = 90, max_gsd: float = 10.0, scale: float = 1000,
                 base_year: float = 0.0):
        self.base_lon, self.base_lat, self.max_gsd, self.scale = base_lon, base_lat, max_gsd, scale
        self.base_year = base_year

    def normalize(self, metadata: Sequence[float]) -> torch.Tensor:
        lon, lat, gsd, year = (float(v) for v in metadata)
        return torch.tensor([lon / (180 + self.base_lon) * self.scale, lat / (90 + self.base_lat) * self.scale,
                             gsd / self.max_gsd * self.scale, year / 2100 * self.scale])

    def unnormalize(self, metadata: Sequence[float], is_print: bool = False) -> torch.Tensor:
        lon, lat, gsd, year = (float(v) for v in metadata)
        return torch.tensor([lon / self.scale * (180 + self.base_lon) - (self.base_lon if is_print else 0),
                             lat / self.scale * (90 + self.base_lat) - (self.base_lat if is_print else 0),
                             gsd / self.scale * self.max_gsd,
                             year / self.scale * 2100 + (self.base_year if is_print else 0)])

    def text_formatting(self, metadata: Sequence[float]) -> str:
        lon, lat, gsd, year = metadata
        s = f" at a resolution of {round(gsd, 5)}. The longitude, latitude is {lon}, {lat}."
        if year != 0.0:
            s += f" The date is {year}."
        return s

    def embedding(self, metadata: Sequence[float]) -> Tuple[torch.Tensor, str]:
        return self.normalize(metadata), self.text_formatting(metadata)


def apply_rotary_emb(x: torch.Tensor, freqs_cis: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]],
                     use_real: bool = True, use_real_unbind_dim: int = -1) -> torch.Tensor:
    """Rotate x [B, H, S, D].  Real form: freqs_cis = (cos, sin) of shape
    [S, D], [B, S, D], [B, 1, S, D] or [B, H, S, D]; pairs are adjacent
    (unbind_dim -1) or split halves (unbind_dim -2).  Complex form:
    freqs_cis [B, S, D/2] complex, pairs adjacent."""
    B, H, S, D = x.shape
    if not use_real:
        xc = torch.view_as_complex(x.float().reshape(B, H, S, D // 2, 2))
        return torch.view_as_real(xc * freqs_cis.unsqueeze(1)).flatten(3).type_as(x)
    cos, sin = freqs_cis
    if cos.dim() == 2:
        cos, sin = cos[None, None], sin[None, None]
    elif cos.dim() == 3:
        cos, sin = cos[:, None], sin[:, None]
    elif cos.dim() == 4:
        if cos.shape[1] not in (1, H):
            raise ValueError(f"4D freqs have {cos.shape[1]} heads, input has {H}")
    else:
        raise ValueError(f"unsupported freqs rank {cos.dim()}")
    cos, sin = cos.to(x.device).float(), sin.to(x.device).float()
    if use_real_unbind_dim == -1:
        re, im = x.float().reshape(B, H, S, D // 2, 2).unbind(-1)
        rot = torch.stack([-im, re], -1).flatten(3)
    elif use_real_unbind_dim == -2:
        re, im = x.float().reshape(B, H, S, 2, D // 2).unbind(-2)
        rot = torch.cat([-im, re], -1)
    else:
        raise ValueError(f"invalid unbind dim {use_real_unbind_dim}")
    return (x.float() * cos + rot * sin).to(x.dtype)


def _trainable_state(model) -> dict:
    return {k: v.detach().contiguous().cpu() for k, v in model.named_parameters()
            if v.requires_grad and "lora_" not in k}


def save_trainable_param_hook(models, weights, output_dir: str, accelerator=None):
    """Save every trainable non-LoRA parameter to <output_dir>/model.safetensors
    (main process only; `accelerator` may be None)."""
    from safetensors.torch import save_file

    if accelerator is not None and not accelerator.is_main_process:
        return
    for model in models:
        m = accelerator.unwrap_model(model) if accelerator is not None else model
        save_file(_trainable_state(m), os.path.join(output_dir, "model.safetensors"))
        if weights:
            weights.pop()


def save_lora_adapter_hook(models, weights, output_dir: str, accelerator=None, target_adapters: List[str] = ()):
    """Save each named LoRA adapter through the model's save_lora_adapter and
    the remaining trainable parameters to model.safetensors."""
    from safetensors.torch import save_file

    if accelerator is not None and not accelerator.is_main_process:
        return
    for model in models:
        m = accelerator.unwrap_model(model) if accelerator is not None else model
        for name in target_adapters:
            m.save_lora_adapter(save_directory=os.path.join(output_dir, name), adapter_name=name)
        sd = _trainable_state(m)
        if sd:
            save_file(sd, os.path.join(output_dir, "model.safetensors"))
        if weights:
            weights.pop()


def encode_images(vae, pixels: torch.Tensor, weight_dtype) -> torch.Tensor:
    z = vae.encode(pixels.to(vae.dtype)).latent_dist.sample()
    return ((z - vae.config.shift_factor) * vae.config.scaling_factor).to(weight_dtype)


@contextmanager
def preserve_requires_grad(model):
    saved = {n: p.requires_grad for n, p in model.named_parameters()}
    try:
        yield
    finally:
        for n, p in model.named_parameters():
            p.requires_grad = saved[n]


@torch.no_grad()
def encode_prompt(prompt: Union[str, List[str]], tokenizer, text_encoder, max_sequence_length: int = 512):
    """Caption embeddings: the chat-templated prompt through the text encoder,
    second-to-last hidden state, padding removed (one [L_i, dim] per prompt)."""
    prompts = [prompt] if isinstance(prompt, str) else list(prompt)
    prompts = [tokenizer.apply_chat_template([{"role": "user", "content": p}], tokenize=False,
                                             add_generation_prompt=True, enable_thinking=True) for p in prompts]
    enc = tokenizer(prompts, padding="max_length", max_length=max_sequence_length, truncation=True,
                    return_tensors="pt")
    dev = text_encoder.device
    ids, mask = enc.input_ids.to(dev), enc.attention_mask.to(dev).bool()
    hid = text_encoder(input_ids=ids, attention_mask=mask, output_hidden_states=True).hidden_states[-2]
    return [hid[i][mask[i]] for i in range(hid.shape[0])]


def load_z_image_text_processer(ckpt_path: str, device, weight_dtype, requires_grad: bool = False):
    from transformers import AutoTokenizer, Qwen3ForCausalLM

    tok = AutoTokenizer.from_pretrained(ckpt_path, subfolder="tokenizer")
    enc = Qwen3ForCausalLM.from_pretrained(ckpt_path, subfolder="text_encoder").to(device, dtype=weight_dtype)
    enc.requires_grad_(requires_grad)
    return tok, enc


class FastInitMode(TorchDispatchMode):
    """Inside this mode every `uniform_` draws from the harp Philox4x32-10
    generator with a fixed seed and a per-call counter offset, so all ranks
    that construct the same model in the same order get identical weights
    without a broadcast (and on the GPU without a host round trip)."""

    def __init__(self, seed: int = 42):
        super().__init__()
        self.seed = seed
        self.calls = 0

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is torch.ops.aten.uniform_.default:
            from ..ops import functional as Fn

            t = args[0]
            lo = float(args[1]) if len(args) > 1 else float(kwargs.get("from", 0.0))
            hi = float(args[2]) if len(args) > 2 else float(kwargs.get("to", 1.0))
            Fn.philox_uniform_(t, self.seed, self.calls << 32, lo, hi)
            self.calls += 1
            return t
        return func(*args, **kwargs)
