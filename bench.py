"""Headline benchmark: DiT training image-tokens/s on N B200 GPUs.

Config ("DiT-XL/2-style training at 1024px"): 28 blocks,
hidden 1152, 16 heads, 2-D RoPE; latent [B, 16, 128, 128] with patch 2
(4096 image tokens) plus 256 text tokens of dim 1152; per-GPU batch 4; bf16;
sequence parallel over all N GPUs; flow-matching loss; AdamW.
Scaling is weak: every GPU always holds 4 samples' worth of tokens
(global batch 4*N split into N sequence chunks), so the GEMM shapes per GPU
are the same at every N.  Weights are random (Philox), data synthetic.

  python bench.py --gpus N --steps K --warmup W [--impl harp|baseline|reference]
  python bench.py --op ring-attn --seq 65536 [--sp-mode ulysses|ring] ...   (attention op sweep)

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
# Measured throughput of the NCCL + cuBLAS/SDPA comparison arm (baseline/,
# `--impl baseline`) for the headline configuration, per GPU count, with the
# commit and date of each measurement; vs_baseline divides by the entry of the
# same GPU count.
BASELINE_FILE = os.path.join(ROOT, "baseline", "measured.json")


def baseline_entry(model: str, n: int):
    try:
        with open(BASELINE_FILE) as fh:
            return json.load(fh).get(model, {}).get(str(n))
    except (OSError, ValueError):
        return None


IMG_TOKENS = 4096
TEXT_TOKENS = 256


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="harp", choices=["harp", "baseline", "reference"])
    ap.add_argument("--model", default="dit-xl-2")
    ap.add_argument("--batch-per-gpu", type=int, default=4,
                    help="dit-*: samples per GPU (weak scaling: each SP group holds batch-per-gpu * sp samples)")
    ap.add_argument("--batch", type=int, default=1, help="mmdit-*/flux-*: samples per SP group (strong scaling)")
    ap.add_argument("--latent", type=int, default=0, help="latent side (default: 128, mmdit-2b 256)")
    ap.add_argument("--text-len", type=int, default=0, help="text tokens (default: 256, flux-12b 512)")
    ap.add_argument("--sp", type=int, default=0, help="sequence-parallel size (default: all GPUs)")
    ap.add_argument("--sp-backend", default="auto", choices=["auto", "torch", "nvl"])
    ap.add_argument("--sp-mode", default="auto", choices=["auto", "ring", "ulysses"],
                    help="sequence-parallel attention: K/V gather (ring) or head all-to-all (ulysses)")
    ap.add_argument("--comm", default="auto", choices=["auto", "torch", "nvl"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--offload-optimizer", action="store_true",
                    help="harp: fp32 master weights and AdamW moments in pinned, mapped host memory "
                         "(the baseline arm does not run this configuration)")
    ap.add_argument("--shard-params", action="store_true",
                    help="harp, N > 1: keep 1/N of every block's weights per GPU and gather them per block; "
                         "baseline: FSDP2 fully_shard per block")
    ap.add_argument("--phases", action="store_true",
                    help="after the timed steps, run --steps more with per-phase CUDA events (forward, backward, "
                         "gradient sync, each sequence-parallel exchange and wait) and print their per-step device "
                         "time, max over ranks, as a second JSON line (implies --cuda-graph 0)")
    ap.add_argument("--cuda-graph", type=int, default=1, choices=[0, 1],
                    help="harp: capture the whole step (on every GPU) in a CUDA graph after two eager warm-up "
                         "steps; the capture itself happens inside the warm-up when --warmup >= 3")
    ap.add_argument("--depth", type=int, default=0, help="override depth (debug only; not a valid bench)")
    ap.add_argument("--op", default="train", choices=["train", "ring-attn"],
                    help="ring-attn: sequence-parallel attention fwd+bwd of Q/K/V [1, 24, seq, 128]")
    ap.add_argument("--seq", type=int, default=16384, help="ring-attn: total sequence length (split over ranks)")
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


def run_ring_attn(args):
    """Sequence-parallel attention forward + backward, Q/K/V [1, 24, S, 128]
    bf16 non-causal, S split evenly over the N ranks (BASELINE.json op sweep).
    harp: fused NVLink Ulysses (head all-to-all inside harp kernels, attention
    consuming chunks as they land) or the NVLink K/V gather ("ring"); baseline:
    NCCL all-gather of K/V + SDPA forward/backward + NCCL reduce-scatter of
    dK/dV.  TFLOP/s of the whole job = 4*S^2*H*D*(1 + 2.5) / time."""
    rank, ws, local = setup_dist(args.gpus)
    device = torch.device("cuda", local)
    B, H, D, S = 1, 24, 128, args.seq
    assert S % ws == 0
    Sl = S // ws
    g = torch.Generator(device=device).manual_seed(17 + rank)
    q, k, v, do = (torch.randn(B * Sl, H * D, device=device, generator=g).to(torch.bfloat16) for _ in range(4))
    mode = "-"
    if args.impl == "harp":
        import harp_b200
        from harp_b200.parallel import sequence as SQ

        assert harp_b200.load_native(build_if_needed=False), "harp CUDA library not built"
        comm = None
        if ws > 1:
            from harp_b200.parallel.nvlink import NVLinkComm

            comm = NVLinkComm.get(dist.group.WORLD, device)
        mode = SQ.resolve_mode(args.sp_mode, H, ws) if ws > 1 else "local"
        sp = SQ.SPContext.from_group(dist.group.WORLD if ws > 1 else None, backend="nvl", comm=comm, mode=mode) \
            if ws > 1 else SQ.SPContext()
        qkv = torch.cat([q, k, v], 1)

        def step():
            if comm is not None:
                comm.begin_step()
                comm.barrier()  # every rank is done with the previous step's buffers
            if SQ.ulysses_nvl(sp):
                o, _, _, saved = comm.uly_forward(qkv, B, Sl, H, D, None, None, None, 0.0, False)
                comm.uly_backward(saved, do, B, Sl, H, D)
            else:
                o, saved = SQ.sp_attention_forward(q, k, v, B, Sl, H, D, sp)
                SQ.sp_attention_backward(saved, q, k, v, o, do, B, Sl, H, D, sp)
    else:
        import torch.nn.functional as F

        def step():
            kv = torch.cat([k, v], 1)
            if ws > 1:
                full = torch.empty(ws * B * Sl, 2 * H * D, device=device, dtype=kv.dtype)
                dist.all_gather_into_tensor(full, kv)
            else:
                full = kv
            kf = full[:, :H * D].reshape(B, S, H, D).transpose(1, 2).detach().requires_grad_(True)
            vf = full[:, H * D:].reshape(B, S, H, D).transpose(1, 2).detach().requires_grad_(True)
            qf = q.view(B, Sl, H, D).transpose(1, 2).detach().requires_grad_(True)
            o = F.scaled_dot_product_attention(qf, kf, vf)
            o.backward(do.view(B, Sl, H, D).transpose(1, 2))
            dkv = torch.cat([kf.grad.transpose(1, 2).reshape(B * S, H * D),
                             vf.grad.transpose(1, 2).reshape(B * S, H * D)], 1)
            if ws > 1:
                mine = torch.empty(B * Sl, 2 * H * D, device=device, dtype=dkv.dtype)
                dist.reduce_scatter_tensor(mine, dkv)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, ws)
    if args.impl == "harp":
        from harp_b200.runtime import errors

        errors.check(device)
    flops = 4.0 * B * H * S * S * D * 3.5
    if rank == 0:
        print(json.dumps({
            "metric": "ring-attn fwd+bwd TFLOPS (whole job, max over ranks)", "value": flops / ms / 1e9,
            "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1) Q/K/V/dO", "impl": args.impl,
            "config": {"op": "sequence-parallel attention fwd+bwd", "q_shape": [B, H, S, D], "seq_total": S,
                       "seq_per_rank": Sl, "causal": False, "mode": mode,
                       "l2": "Q/K/V/dO per rank %.0f MB; K/V of all ranks %.0f MB" %
                             (4 * B * Sl * H * D * 2 / 1e6, 2 * B * S * H * D * 2 / 1e6)},
        }), flush=True)
    if ws > 1:
        if args.impl == "harp":
            from harp_b200.parallel.nvlink import NVLinkComm

            torch.cuda.synchronize()
            NVLinkComm.close_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.phases:
        args.cuda_graph = 0
    if args.impl == "reference":
        return run_reference(args)
    if args.op == "ring-attn":
        return run_ring_attn(args)
    from harp_b200.models.dit import PRESETS as _DIT_PRESETS

    family = "dit" if args.model in _DIT_PRESETS else "mmdit"
    weak = args.model.startswith("dit") or args.model in ("tiny", "small")
    args.latent = args.latent or (256 if args.model == "mmdit-2b" else 128)
    args.text_len = args.text_len or (512 if args.model == "flux-12b" else TEXT_TOKENS)
    img_tokens = (args.latent // 2) ** 2
    if args.impl == "baseline" and args.model == "flux-12b":
        # FSDP2 raised an illegal memory access on this pool's B200s for this
        # model (with and without CPU offload); that configuration is not run
        print(json.dumps({"impl": "baseline", "unavailable": "the baseline's FSDP2 run of flux-12b is not run on "
                          "this pool (it raised an illegal memory access in library code)"}))
        return 0
    if args.impl == "baseline" and args.offload_optimizer:
        # FSDP2's CPUOffloadPolicy raised an illegal memory access on this pool's
        # B200s (flux-12b, 2 GPUs); that configuration is not run
        print(json.dumps({"impl": "baseline", "unavailable": "the baseline's FSDP2 CPU-offload configuration is "
                          "not run on this pool (it raised an illegal memory access); use --shard-params alone"}))
        return 0
    rank, ws, local = setup_dist(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sp = args.sp or ws
    # dit: weak scaling, each GPU holds batch_per_gpu samples' worth of tokens;
    # mmdit/flux: a fixed batch per SP group split over its ranks (strong scaling)
    B = args.batch_per_gpu * sp if weak else args.batch
    dp = ws // sp
    global_batch = B * dp

    if args.impl == "harp":
        import harp_b200
        from harp_b200.trainer import ParallelState, TrainConfig, Trainer

        assert harp_b200.load_native(build_if_needed=False), "harp CUDA library not built (run __graft_entry__.build())"
        par = ParallelState.build(sp)
        if family == "dit":
            from harp_b200.models.dit import DiT, PRESETS

            cfg = PRESETS[args.model]
            if args.depth:
                import dataclasses

                cfg = dataclasses.replace(cfg, depth=args.depth)
            with torch.device(device):
                model = DiT(cfg)
            loss_fn = None
        else:
            from harp_b200.models import mmdit as M

            cfg = M.PRESETS[args.model]
            if args.depth:
                import dataclasses

                cfg = dataclasses.replace(cfg, depth_double=min(cfg.depth_double, args.depth),
                                          depth_single=min(cfg.depth_single, args.depth))
            with torch.device(device):
                model = M.MMDiT(cfg)
            loss_fn = M.mmdit_loss_local
        model.initialize_weights(seed=0)
        model = model.to(torch.bfloat16)
        trainer = Trainer(model, par, TrainConfig(comm=args.comm, cuda_graph=bool(args.cuda_graph),
                                                  shard_params=args.shard_params and ws > 1,
                                                  offload_optimizer=args.offload_optimizer), device,
                          sp_backend=args.sp_backend, sp_mode=args.sp_mode, loss_fn=loss_fn)
        cin, tdim = cfg.in_channels, cfg.text_dim

        def step(b):
            return trainer.run(b)

        def e2e_step(b):
            return trainer.step(b)

        count_launches = lambda: int(torch.ops.harp.launch_count())  # noqa: E731
        reset_launches = lambda: torch.ops.harp.reset_launch_count()  # noqa: E731
        parallelism = (f"sp{sp}" + (f"xdp{dp}" if dp > 1 else "") + (f"-{trainer.sp.mode}" if sp > 1 else "") +
                       ("-sharded-weights" if trainer.gatherer is not None else "") +
                       ("-offload-optimizer" if args.offload_optimizer else ""))
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        if family == "dit":
            from baseline.dit_baseline import BaselineTrainer

            trainer = BaselineTrainer(args.model, device, sp, depth=args.depth or None)
        else:
            from baseline.mmdit_baseline import BaselineMMDiTTrainer

            trainer = BaselineMMDiTTrainer(args.model, device, sp, depth=args.depth or None,
                                           shard=args.shard_params, offload=args.offload_optimizer)
        cin, tdim = trainer.cfg.in_channels, trainer.cfg.text_dim

        def step(b):
            return trainer.train_step(b["latent"], b["noise"], b["text"], b["sigmas"])

        e2e_step = trainer.step
        count_launches = lambda: 0  # noqa: E731
        reset_launches = lambda: None  # noqa: E731
        parallelism = (f"sp{sp}" + (f"xdp{dp}" if dp > 1 else "") +
                       ("-fsdp2" if getattr(trainer, "shard", False) else "") +
                       ("-cpu-offload" if getattr(trainer, "shard", False) and args.offload_optimizer else ""))

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
    value = global_batch * img_tokens / (ms / 1000.0)

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
        e2e = {"value": global_batch * img_tokens / (el / args.steps), "unit": "image-tokens/s",
               "ms_per_step": 1000.0 * el / args.steps, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "api": "Trainer.step" if args.impl == "harp" else "BaselineTrainer.step", "last_loss": last}

    headline = (args.model == "dit-xl-2" and not args.depth and weak and args.batch_per_gpu == 4 and
                args.latent == 128 and args.text_len == TEXT_TOKENS and sp == ws)
    base = baseline_entry(args.model, ws) if headline and args.impl == "harp" else None
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
            "scaling": "weak" if weak else "strong",
            "vs_baseline": (value / base["value"] if base else None),
            "baseline_source": ({k: base[k] for k in ("value", "commit", "date") if k in base} if base else None),
            "dtype": "bf16",
            "data": "synthetic (random latents/text embeddings of the named shapes, random-init weights)",
            "impl": args.impl,
            "config": {
                "model": args.model if not args.depth else f"{args.model}(depth={args.depth}, NOT VALID)",
                "global_batch": global_batch,
                "per_gpu_batch": args.batch_per_gpu if weak else global_batch / ws,
                "seq_len": img_tokens + args.text_len,
                "image_tokens": img_tokens,
                "text_tokens": args.text_len,
                "latent": [16, args.latent, args.latent],
                "parallelism": parallelism,
                "cuda_graph": bool(getattr(trainer, "graph_enabled", False)),
                "l2": "inputs larger than L2 (weights %.1f GB, activations > 10 GB per step)" %
                      (sum(p.numel() for p in trainer.model.parameters()) * 2 / 1e9 if args.impl == "harp"
                       else sum(p.numel() for p in trainer.params) * 2 / 1e9 if hasattr(trainer, "params")
                       else 1.35),
            },
            "loss": float(loss.reshape(-1)[0].item()),
            "gpu_launches": launches,
            "clocks": clocks,
            "e2e": e2e,
        }
        print(json.dumps(out), flush=True)
    if args.phases and args.impl == "harp":
        from harp_b200.utils import observability as obs

        timer = obs.enable_phases(True)
        for _ in range(args.steps):
            step(dev_batch)
        rep = timer.report()  # syncs; max over ranks
        obs.enable_phases(False)
        if rank == 0:
            print(json.dumps({"phases_ms_per_step": {k: round(v / args.steps, 3) for k, v in sorted(rep.items())},
                              "n_gpus": ws, "steps": args.steps, "ms_per_step_timed": ms,
                              "note": "CUDA events on the launching stream, summed per step, max over ranks; "
                                      "nested phases (uly.*) are inside forward/backward"}), flush=True)
    if args.impl == "harp":
        torch.cuda.synchronize()
        trainer.close()  # a captured step holding NCCL work goes before the process group
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
