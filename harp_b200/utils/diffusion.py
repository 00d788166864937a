"""Flow-matching training utilities: scheduler, timestep density, loss
weighting and learning-rate schedules.

Semantics follow the reference's src/utils/standalone_diffusion.py:
  FlowMatchEulerDiscreteScheduler   :23-89  (timesteps N..1, sigmas = t/N with
                                             the static shift s*sig/(1+(s-1)*sig))
  LR schedules                      :92-250 (constant, constant_with_warmup,
                                             linear, cosine, cosine_with_restarts,
                                             polynomial, piecewise_constant)
  compute_density_for_timestep_sampling   :253-270
  compute_loss_weighting_for_sd3          :273-281
"""
from __future__ import annotations

import json
import math
import os
from typing import Sequence, Optional, Union

import torch
from torch.optim import Optimizer
from torch.optim.lr_scheduler import LambdaLR


class _Config(dict):
    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e


class FlowMatchEulerDiscreteScheduler:
    config_name = "scheduler_config.json"
    order = 1

    def __init__(self, num_train_timesteps: int = 1000, shift: float = 1.0, use_dynamic_shifting: bool = False,
                 base_shift: Optional[float] = 0.5, max_shift: Optional[float] = 1.15,
                 base_image_seq_len: Optional[int] = 256, max_image_seq_len: Optional[int] = 4096,
                 invert_sigmas: bool = False, **extra):
        self.config = _Config(num_train_timesteps=num_train_timesteps, shift=shift,
                              use_dynamic_shifting=use_dynamic_shifting, base_shift=base_shift, max_shift=max_shift,
                              base_image_seq_len=base_image_seq_len, max_image_seq_len=max_image_seq_len,
                              invert_sigmas=invert_sigmas, **extra)
        t = torch.linspace(num_train_timesteps, 1, num_train_timesteps, dtype=torch.float32)
        sig = t / num_train_timesteps
        if not use_dynamic_shifting:
            sig = shift * sig / (1 + (shift - 1) * sig)
        self.sigmas = sig
        self.timesteps = sig * num_train_timesteps
        self.sigma_min = float(sig[-1])
        self.sigma_max = float(sig[0])

    @classmethod
    def from_pretrained(cls, path: str, subfolder: Optional[str] = None):
        p = os.path.expanduser(path)
        if subfolder:
            p = os.path.join(p, subfolder)
        if os.path.isdir(p):
            p = os.path.join(p, cls.config_name)
        if not os.path.exists(p):
            return cls()
        with open(p) as fh:
            return cls(**json.load(fh))

    def save_config(self, directory: str):
        os.makedirs(directory, exist_ok=True)
        with open(os.path.join(directory, self.config_name), "w") as fh:
            json.dump(dict(self.config), fh, indent=2)

    # -- sampling (inference) --------------------------------------------------
    @staticmethod
    def time_shift(mu: float, sigma: torch.Tensor) -> torch.Tensor:
        """Resolution-dependent shift e^mu / (e^mu + 1/sigma - 1) (SD3 / Flux)."""
        return math.exp(mu) / (math.exp(mu) + (1.0 / sigma - 1.0))

    def set_timesteps(self, num_inference_steps: Optional[int] = None, device=None,
                      sigmas: Optional[Sequence[float]] = None, mu: Optional[float] = None,
                      timesteps: Optional[Sequence[float]] = None):
        """Sampling grid: `num_inference_steps` sigmas from sigma_max down to
        sigma_min (or the given sigmas / timesteps), shifted (static `shift`, or
        time_shift(mu) with dynamic shifting), followed by a terminal 0."""
        n_train = self.config.num_train_timesteps
        if sigmas is not None:
            sig = torch.tensor(list(sigmas), dtype=torch.float64)
        elif timesteps is not None:
            sig = torch.tensor(list(timesteps), dtype=torch.float64) / n_train
        else:
            sig = torch.linspace(self.sigma_max * n_train, self.sigma_min * n_train, num_inference_steps,
                                 dtype=torch.float64) / n_train
        if self.config.use_dynamic_shifting:
            if mu is None:
                raise ValueError("dynamic shifting needs mu")
            sig = self.time_shift(mu, sig.clamp_min(1e-12))
        else:
            s = self.config.shift
            sig = s * sig / (1 + (s - 1) * sig)
        self.num_inference_steps = len(sig)
        self.timesteps = (sig * n_train).float().to(device or "cpu")
        self.sigmas = torch.cat([sig, sig.new_zeros(1)]).float().to(device or "cpu")
        self._step_index = 0

    def step(self, model_output: torch.Tensor, timestep, sample: torch.Tensor, return_dict: bool = False):
        """Euler step of dx/dsigma = model_output (the noise - x0 velocity)."""
        i = self._step_index
        s, s_next = self.sigmas[i], self.sigmas[i + 1]
        prev = (sample.float() + (s_next - s).to(sample.device) * model_output.float()).to(sample.dtype)
        self._step_index += 1
        return (prev,) if not return_dict else {"prev_sample": prev}

    def sigmas_for(self, timesteps: torch.Tensor) -> torch.Tensor:
        """sigma of each (exact) training timestep value."""
        idx = torch.searchsorted(-self.timesteps, -timesteps.float().cpu())
        idx = idx.clamp(0, len(self.sigmas) - 1)
        return self.sigmas[idx]


def compute_density_for_timestep_sampling(weighting_scheme: str, batch_size: int, logit_mean: float = 0.0,
                                          logit_std: float = 1.0, mode_scale: float = 1.29,
                                          device: Union[torch.device, str] = "cpu",
                                          generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """u in [0, 1) from which timestep indices are drawn."""
    if weighting_scheme == "logit_normal":
        u = torch.normal(mean=logit_mean, std=logit_std, size=(batch_size,), device=device, generator=generator)
        return torch.sigmoid(u)
    u = torch.rand(size=(batch_size,), device=device, generator=generator)
    if weighting_scheme == "mode":
        u = 1 - u - mode_scale * (torch.cos(math.pi * u / 2) ** 2 - 1 + u)
    return u


def compute_loss_weighting_for_sd3(weighting_scheme: str, sigmas: torch.Tensor) -> torch.Tensor:
    if weighting_scheme == "sigma_sqrt":
        return (sigmas ** -2.0).float()
    if weighting_scheme == "cosmap":
        bot = 1 - 2 * sigmas + 2 * sigmas ** 2
        return 2 / (math.pi * bot)
    return torch.ones_like(sigmas)


# ---------------------------------------------------------------------------
# learning-rate schedules
# ---------------------------------------------------------------------------
def _warm(step, warmup):
    return float(step) / float(max(1, warmup))


def get_scheduler(name: str, optimizer: Optimizer, step_rules: Optional[str] = None,
                  num_warmup_steps: Optional[int] = None, num_training_steps: Optional[int] = None,
                  num_cycles: Union[int, float] = 1, power: float = 1.0, lr_end: float = 1e-7,
                  last_epoch: int = -1) -> LambdaLR:
    name = name.lower()
    if name not in ("constant", "piecewise_constant") and num_warmup_steps is None:
        raise ValueError(f"{name} requires num_warmup_steps")
    W = num_warmup_steps or 0
    T = num_training_steps

    if name == "constant":
        fn = lambda s: 1.0  # noqa: E731
    elif name == "constant_with_warmup":
        fn = lambda s: _warm(s, W) if s < W else 1.0  # noqa: E731
    elif name == "piecewise_constant":
        rules = {}
        parts = (step_rules or "1").split(",")
        for r in parts[:-1]:
            v, st = r.split(":")
            rules[int(st)] = float(v)
        last = float(parts[-1])

        def fn(s):
            for k in sorted(rules):
                if s < k:
                    return rules[k]
            return last
    else:
        if T is None:
            raise ValueError(f"{name} requires num_training_steps")
        if name == "linear":
            def fn(s):
                if s < W:
                    return _warm(s, W)
                return max(0.0, float(T - s) / float(max(1, T - W)))
        elif name == "cosine":
            def fn(s):
                if s < W:
                    return _warm(s, W)
                prog = float(s - W) / float(max(1, T - W))
                return max(0.0, 0.5 * (1.0 + math.cos(math.pi * 0.5 * 2.0 * prog)))
        elif name == "cosine_with_restarts":
            def fn(s):
                if s < W:
                    return _warm(s, W)
                prog = float(s - W) / float(max(1, T - W))
                if prog >= 1.0:
                    return 0.0
                return max(0.0, 0.5 * (1.0 + math.cos(math.pi * ((float(num_cycles) * prog) % 1.0))))
        elif name == "polynomial":
            lr_init = optimizer.defaults["lr"]
            if not lr_init > lr_end:
                raise ValueError("lr_end must be smaller than the initial lr")

            def fn(s):
                if s < W:
                    return _warm(s, W)
                if s > T:
                    return lr_end / lr_init
                rem = 1 - (s - W) / max(1, T - W)
                return ((lr_init - lr_end) * rem ** power + lr_end) / lr_init
        else:
            raise ValueError(f"unknown lr scheduler {name}")
    return LambdaLR(optimizer, fn, last_epoch)


class LRSchedule:
    """Learning-rate schedule for optimizers that are not torch.optim
    (the sharded AdamW): same multipliers as get_scheduler."""

    def __init__(self, name: str, base_lr: float, **kw):
        dummy = torch.optim.SGD([torch.zeros(1, requires_grad=True)], lr=base_lr)
        self._sched = get_scheduler(name, dummy, **kw)
        self._opt = dummy

    def lr(self) -> float:
        return self._opt.param_groups[0]["lr"]

    def step(self):
        self._opt.step()
        self._sched.step()

    def state_dict(self):
        return self._sched.state_dict()

    def load_state_dict(self, sd):
        self._sched.load_state_dict(sd)
        self._opt.param_groups[0]["lr"] = self._sched.get_last_lr()[0]
