"""Headline benchmark: DiT training image-tokens/s on N B200 GPUs.

Config ("DiT-XL/2-style training at 1024px"): 28 blocks,
hidden 1152, 16 heads, 2-D RoPE; latent [B, 16, 128, 128] with patch 2
(4096 image tokens) plus 256 text tokens of dim 1152; per-GPU batch 4; bf16;
sequence parallel over all N GPUs; flow-matching loss; AdamW.
Scaling is weak: every GPU always holds 4 samples' worth of tokens
(global batch 4*N split into N sequence chunks), so the GEMM shapes per GPU
are the same at every N.  Weights are random (Philox), data synthetic.

  python bench.py --gpus N --steps K --warmup W [--impl harp|baseline|reference]

N > 1 is launched by torchrun (RANK / LOCAL_RANK / WORLD_SIZE from the env).
Rank 0 prints one JSON line.  `value` is device-timed (CUDA events on the
compute stream, barrier + synchronize on both sides, max over ranks) with
inputs resident on the GPU; `e2e` is the same metric through the public API
(Trainer.step: pinned host batch -> GPU copy -> step -> loss.item()).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "DiT train image-tokens/sec (max over ranks)"
IMG_TOKENS = 4096
TEXT_TOKENS = 256


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="harp", choices=["harp", "baseline", "reference"])
    ap.add_argument("--model", default="dit-xl-2")
    ap.add_argument("--batch-per-gpu", type=int, default=4)
    ap.add_argument("--latent", type=int, default=128)
    ap.add_argument("--text-len", type=int, default=TEXT_TOKENS)
    ap.add_argument("--sp", type=int, default=0, help="sequence-parallel size (default: all GPUs)")
    ap.add_argument("--sp-backend", default="auto", choices=["auto", "torch", "nvl"])
    ap.add_argument("--sp-mode", default="auto", choices=["auto", "ring", "ulysses"],
                    help="sequence-parallel attention: K/V gather (ring) or head all-to-all (ulysses)")
    ap.add_argument("--comm", default="auto", choices=["auto", "torch", "nvl"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--depth", type=int, default=0, help="override depth (debug only; not a valid bench)")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.proc is None:
            return out
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            rows = [l.split(",") for l in open(self.path).read().strip().splitlines() if l.strip()]
        except Exception:
            rows = []
        clocks, maxc, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                clocks.append(float(r[1]))
                maxc.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if clocks:
            out["sm_mhz"] = statistics.median(clocks)
            out["sm_max_mhz"] = max(maxc)
        out["reasons"] = sorted(reasons)
        out["samples"] = len(clocks)
        return out


def setup_dist(n_gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        import datetime

        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
        return dist.get_rank(), ws, local
    return 0, 1, 0


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_batch(B, C, L, text_len, text_dim, device, seed, pinned=False):
    g = torch.Generator().manual_seed(seed)
    batch = {
        "latent": torch.randn(B, C, L, L, generator=g).to(torch.bfloat16),
        "noise": torch.randn(B, C, L, L, generator=g).to(torch.bfloat16),
        "text": torch.randn(B, text_len, text_dim, generator=g).to(torch.bfloat16),
        "sigmas": torch.rand(B, generator=g),
    }
    if pinned:
        return {k: v.pin_memory() for k, v in batch.items()}
    return {k: v.to(device) for k, v in batch.items()}


def run_reference(args):
    why = ("pip install of the reference fails: 'Directory is not installable. Neither setup.py nor "
           "pyproject.toml found'; it is a CPU-only ARMv9 SME/SVE stack needing the "
           "-march=armv9+sve+sve2+sme toolchain, HMPI and KBLAS, and its kernels/_C*.so op library is not "
           "shipped, so it can neither be installed nor run on a B200 box")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}))
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    rank, ws, local = setup_dist(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sp = args.sp or ws
    B = args.batch_per_gpu * sp  # per SP group; each GPU holds B * S / sp tokens = 4 samples' worth
    dp = ws // sp
    global_batch = B * dp

    if args.impl == "harp":
        import harp_b200
        from harp_b200.models.dit import DiT, PRESETS
        from harp_b200.trainer import ParallelState, TrainConfig, Trainer

        assert harp_b200.load_native(build_if_needed=False), "harp CUDA library not built (run __graft_entry__.build())"
        cfg = PRESETS[args.model]
        if args.depth:
            import dataclasses

            cfg = dataclasses.replace(cfg, depth=args.depth)
        par = ParallelState.build(sp)
        with torch.device(device):
            model = DiT(cfg)
        model.initialize_weights(seed=0)
        model = model.to(torch.bfloat16)
        trainer = Trainer(model, par, TrainConfig(comm=args.comm), device, sp_backend=args.sp_backend,
                          sp_mode=args.sp_mode)
        cin, tdim = cfg.in_channels, cfg.text_dim

        def step(b):
            return trainer.train_step(b["latent"], b["noise"], b["text"], b["sigmas"])

        def e2e_step(b):
            return trainer.step(b)

        count_launches = lambda: int(torch.ops.harp.launch_count())  # noqa: E731
        reset_launches = lambda: torch.ops.harp.reset_launch_count()  # noqa: E731
        parallelism = f"sp{sp}" + (f"xdp{dp}" if dp > 1 else "") + (f"-{trainer.sp.mode}" if sp > 1 else "")
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from baseline.dit_baseline import BaselineTrainer

        trainer = BaselineTrainer(args.model, device, sp, depth=args.depth or None)
        cin, tdim = trainer.cfg.in_channels, trainer.cfg.text_dim

        def step(b):
            return trainer.train_step(b["latent"], b["noise"], b["text"], b["sigmas"])

        e2e_step = trainer.step
        count_launches = lambda: 0  # noqa: E731
        reset_launches = lambda: None  # noqa: E731
        parallelism = f"sp{sp}" + (f"xdp{dp}" if dp > 1 else "")

    dp_rank = rank // sp
    dev_batch = make_batch(B, cin, args.latent, args.text_len, tdim, device, seed=1234 + dp_rank)
    for _ in range(args.warmup):
        step(dev_batch)
    torch.cuda.synchronize()
    if args.impl == "harp":
        trainer.check_errors()

    sampler = ClockSampler([local] if ws == 1 else list(range(ws))) if rank == 0 else None
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    reset_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(args.steps):
        loss = step(dev_batch)
    ev1.record()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    launches = count_launches()
    clocks = sampler.stop() if sampler else None
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms, ws)
    if args.impl == "harp":
        trainer.check_errors()
    value = global_batch * IMG_TOKENS / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        host_batch = make_batch(B, cin, args.latent, args.text_len, tdim, device, seed=99 + dp_rank, pinned=True)
        e2e_step(host_batch)
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            last = e2e_step(host_batch)
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        el = max_over_ranks(el, ws)
        h2d = sum(v.numel() * v.element_size() for v in host_batch.values())
        e2e = {"value": global_batch * IMG_TOKENS / (el / args.steps), "unit": "image-tokens/s",
               "ms_per_step": 1000.0 * el / args.steps, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "api": "Trainer.step" if args.impl == "harp" else "BaselineTrainer.step", "last_loss": last}

    if rank == 0:
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "image-tokens/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random latents/text embeddings of the named shapes, random-init weights)",
            "impl": args.impl,
            "config": {
                "model": args.model if not args.depth else f"{args.model}(depth={args.depth}, NOT VALID)",
                "global_batch": global_batch,
                "per_gpu_batch": args.batch_per_gpu,
                "seq_len": IMG_TOKENS + args.text_len,
                "image_tokens": IMG_TOKENS,
                "text_tokens": args.text_len,
                "latent": [16, args.latent, args.latent],
                "parallelism": parallelism,
                "l2": "inputs larger than L2 (weights 1.7 GB, activations > 10 GB per step)",
            },
            "loss": float(loss.reshape(-1)[0].item()),
            "gpu_launches": launches,
            "clocks": clocks,
            "e2e": e2e,
        }
        print(json.dumps(out), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
