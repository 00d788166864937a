"""Training entry point (reference: train.py).

Same flags and step semantics as the reference's training driver, on the
harp_b200 engine:

  torchrun --nproc-per-node 8 train.py --model zimage-6b --data_root data/ --sp_size 8
  torchrun --nproc-per-node 8 train.py --model dit-xl-2 --synthetic --sp_size 8
  mpirun -np 8 python train.py ...   (ranks from OMPI_COMM_WORLD_*, as the reference)

Per step (train.py:454-537 of the reference): sample u from the timestep
density, pick the scheduler timesteps and sigmas, x_t = (1 - s) x0 + s eps,
forward the sequence-parallel model, weighted MSE flow-matching loss (divided
by the data-parallel size), backward, gradient reduce-scatter + AdamW +
parameter all-gather, LR-schedule step, logging, checkpoint every
--checkpointing_steps.  Fixes relative to the reference: samples are drawn by
data-parallel rank (SP ranks of a group see the same sample), weight decay is
applied, checkpoints hold the weights and every optimizer shard, and resume
works.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time
from datetime import datetime as _dt

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="harp_b200 training")
    p.add_argument("--pretrained_model_name_or_path", type=str, default="",
                   help="directory with transformer/config.json and scheduler/scheduler_config.json")
    p.add_argument("--model", type=str, default="dit-xl-2",
                   help="dit-xl-2 | mmdit-2b | tiny | small (joint DiT) | zimage-6b | zimage-tiny | sd3-2b | mmdit-tiny | "
             "flux-12b | flux-tiny (double-stream)")
    p.add_argument("--work_dir", type=str, default="work_dir")
    p.add_argument("--sub_work_dir", type=str, default="")
    p.add_argument("--data_root", type=str, default="", help="index.json of .npz samples (empty: synthetic)")
    p.add_argument("--synthetic", action="store_true")
    p.add_argument("--latent_size", type=int, default=128)
    p.add_argument("--text_len", type=int, default=256)
    p.add_argument("--checkpointing_steps", type=int, default=4000)
    p.add_argument("--resume_from_checkpoint", type=str, default=None)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--train_batch_size", type=int, default=1, help="samples per SP group per step")
    p.add_argument("--num_train_epochs", type=int, default=None)
    p.add_argument("--max_train_steps", type=int, default=60000)
    p.add_argument("--learning_rate", type=float, default=1e-4)
    p.add_argument("--scale_lr", action="store_true", default=False)
    p.add_argument("--lr_scheduler", type=str, default="cosine",
                   choices=["linear", "cosine", "cosine_with_restarts", "polynomial", "constant",
                            "constant_with_warmup"])
    p.add_argument("--lr_warmup_steps", type=int, default=500)
    p.add_argument("--weighting_scheme", type=str, default="none",
                   choices=["sigma_sqrt", "logit_normal", "mode", "cosmap", "none"])
    p.add_argument("--logit_mean", type=float, default=0.0)
    p.add_argument("--logit_std", type=float, default=1.0)
    p.add_argument("--mode_scale", type=float, default=1.29)
    p.add_argument("--dataloader_num_workers", type=int, default=0)
    p.add_argument("--adam_beta1", type=float, default=0.9)
    p.add_argument("--adam_beta2", type=float, default=0.999)
    p.add_argument("--adam_weight_decay", type=float, default=1e-2)
    p.add_argument("--adam_epsilon", type=float, default=1e-8)
    p.add_argument("--max_grad_norm", default=1.0, type=float, help="accepted; not applied (as in the reference)")
    p.add_argument("--log_interval", type=int, default=1)
    p.add_argument("--sp_size", type=int, default=4)
    p.add_argument("--rs_size", type=int, default=16, help="RS group size (rows of a parameter; the managers API); the trainer shards its optimizer over every rank")
    p.add_argument("--comm_backend", type=str, default="auto", choices=["auto", "nvl", "torch"])
    p.add_argument("--sp_mode", type=str, default="auto", choices=["auto", "ring", "ulysses"],
                   help="sequence-parallel attention: K/V gather (the reference's ring) or head all-to-all")
    p.add_argument("--enable_profiler", action="store_true")
    p.add_argument("--cuda_graph", action="store_true",
                   help="capture the whole training step in one CUDA graph after two eager steps "
                        "(1 GPU, or N GPUs on the NVLink communicator)")
    p.add_argument("--harp_block_compat", action="store_true", help="Z-Image: reproduce HARP's block residual")
    p.add_argument("--gradient_checkpointing", action="store_true",
                   help="Z-Image: recompute each block's activations in the backward instead of keeping them")
    # accepted for command-line compatibility, unused (as in the reference)
    for flag, typ, default in (("--use_8bit_adam", bool, False), ("--rank", int, 8), ("--resolution", int, 512),
                               ("--cache_dir", str, "cache"), ("--comp_ckpt", str, None)):
        p.add_argument(flag, type=typ, default=default)
    args = p.parse_args(argv)
    if args.sub_work_dir:
        args.work_dir = os.path.join(args.work_dir, args.sub_work_dir)
    args.run_timestamp = _dt.now().strftime("%y_%m_%d-%H:%M:%S")
    return args


def discover_ranks():
    """torchrun (RANK/WORLD_SIZE/LOCAL_RANK) or mpirun (OMPI_COMM_WORLD_*)."""
    env = os.environ
    if "OMPI_COMM_WORLD_RANK" in env and "RANK" not in env:
        env["RANK"] = env["OMPI_COMM_WORLD_RANK"]
        env["WORLD_SIZE"] = env["OMPI_COMM_WORLD_SIZE"]
        env["LOCAL_RANK"] = env.get("OMPI_COMM_WORLD_LOCAL_RANK", env["OMPI_COMM_WORLD_RANK"])
        env.setdefault("MASTER_ADDR", "127.0.0.1")
        env.setdefault("MASTER_PORT", "29500")
    return int(env.get("RANK", 0)), int(env.get("WORLD_SIZE", 1)), int(env.get("LOCAL_RANK", 0))


def build_model(args, device, sp_group, dtype=torch.bfloat16):
    """Returns (model, loss_fn, data shapes)."""
    name = args.model
    if name.startswith("zimage"):
        from harp_b200.models import zimage as Z

        if args.pretrained_model_name_or_path:
            cfg = Z.ZImageTransformer2DModel.load_config(args.pretrained_model_name_or_path, subfolder="transformer")
        else:
            cfg = Z.PRESETS[name]
        with torch.device(device):
            base = Z.ZImageTransformer2DModel.from_config(cfg)
            model = Z.Z_Transformer(base, num_metadata=4, use_cond=True, sp_group_model=sp_group,
                                    harp_block_compat=args.harp_block_compat)
        model = model.to(dtype)
        _init_fixed(model, args.seed)
        if getattr(args, "gradient_checkpointing", False):
            model.gradient_checkpointing_enable()
        shapes = dict(C=base.in_channels, cap_dim=cfg.get("cap_feat_dim", 2560), kind="zimage")

        def loss_fn(m, latent, noise, text, sigmas, sp, weighting=None, metadata=None, cond=None):
            return Z.zimage_loss_local(m, latent, noise, text, sigmas, sp, metadata=metadata, cond=cond,
                                       weighting=weighting)

        return model, loss_fn, shapes
    from harp_b200.models import mmdit as M

    if name in M.PRESETS:
        cfg = M.PRESETS[name]
        with torch.device(device):
            model = M.MMDiT(cfg)
        model.initialize_weights(args.seed)
        model = model.to(dtype)
        shapes = dict(C=cfg.in_channels, cap_dim=cfg.text_dim, kind="mmdit")
        return model, M.mmdit_loss_local, shapes
    from harp_b200.models.dit import PRESETS, DiT, flow_matching_loss_local

    cfg = PRESETS[name]
    with torch.device(device):
        model = DiT(cfg)
    model.initialize_weights(args.seed)
    model = model.to(dtype)

    def loss_fn(m, latent, noise, text, sigmas, sp, weighting=None, **_):
        return flow_matching_loss_local(m, latent, noise, text, sigmas, sp, weighting=weighting)

    return model, loss_fn, dict(C=cfg.in_channels, cap_dim=cfg.text_dim, kind="dit")


@torch.no_grad()
def _init_fixed(model, seed):
    """Identical initial weights on every rank, drawn with Philox per parameter
    (the reference's FastInitMode, train.py:274-285)."""
    from harp_b200.ops import functional as Fn

    for i, (name, p) in enumerate(model.named_parameters()):
        if "norm" in name:
            p.fill_(1.0)
        elif name.endswith("bias") or "pad_token" in name:
            p.zero_()
        else:
            fan_in = p.shape[-1] if p.dim() > 1 else p.numel()
            bound = 1.0 / math.sqrt(max(1, fan_in))
            Fn.philox_uniform_(p.data, seed, i << 32, -bound, bound)


def main(args):
    from harp_b200.runtime import errors
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer
    from harp_b200.utils import diffusion as D
    from harp_b200.utils.checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
    from harp_b200.utils.data import NpzDataset, SyntheticDiTData, collate
    from harp_b200.utils.fault import FaultInjector
    from harp_b200.utils.observability import JsonlWriter, PhaseTimer, make_profiler, setup_logger

    rank, world, local = discover_ranks()
    if os.environ.get("HARP_BIND_CPUS") == "1":
        from harp_b200.launch import bind_process

        bind_process(local)
    use_cuda = torch.cuda.is_available()
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
        import harp_b200

        if not harp_b200.load_native(build_if_needed=True):
            raise RuntimeError("harp_b200 CUDA library is required on GPUs")
    if world > 1:
        backend = "nccl" if use_cuda else "gloo"
        kw = {"device_id": device} if use_cuda else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(minutes=10), **kw)
        # one run directory for all ranks: rank 0's start time (the ranks parse
        # their arguments at different moments, possibly in different seconds)
        stamp = [args.run_timestamp]
        dist.broadcast_object_list(stamp, src=0)
        args.run_timestamp = stamp[0]
    sp_size = min(args.sp_size, world) if world > 1 else 1
    par = ParallelState.build(sp_size, args.rs_size)
    is_main = rank == 0
    args.work_dir = os.path.join(args.work_dir, args.run_timestamp) if not args.resume_from_checkpoint else \
        args.work_dir
    if is_main:
        os.makedirs(args.work_dir, exist_ok=True)
        with open(os.path.join(args.work_dir, "config.json"), "w") as fh:
            json.dump(vars(args), fh, indent=2)
    log = setup_logger(os.path.join(args.work_dir, "train.log"), is_main)
    dp_rank = rank // par.sp_size
    torch.manual_seed(args.seed + dp_rank)
    fault = FaultInjector(rank=rank)

    model, loss_fn, shapes = build_model(args, device, par.sp_group)
    lr = args.learning_rate * (world * args.train_batch_size if args.scale_lr else 1)
    tcfg = TrainConfig(lr=lr, beta1=args.adam_beta1, beta2=args.adam_beta2, eps=args.adam_epsilon,
                       weight_decay=args.adam_weight_decay, comm=args.comm_backend,
                       cuda_graph=bool(getattr(args, "cuda_graph", False)))
    trainer = Trainer(model, par, tcfg, device, sp_backend=args.comm_backend, loss_fn=loss_fn,
                      sp_mode=args.sp_mode)
    sched = D.FlowMatchEulerDiscreteScheduler.from_pretrained(args.pretrained_model_name_or_path or ".",
                                                              subfolder="scheduler")
    lrs = D.LRSchedule(args.lr_scheduler, lr, num_warmup_steps=args.lr_warmup_steps,
                       num_training_steps=args.max_train_steps)

    # data: sampled by data-parallel rank so all SP ranks of a group see the same samples
    if args.data_root and not args.synthetic:
        ds = NpzDataset(args.data_root)
    else:
        ds = SyntheticDiTData(max(64, args.max_train_steps * args.train_batch_size), shapes["C"], args.latent_size,
                              args.text_len, shapes["cap_dim"], num_metadata=4 if shapes["kind"] == "zimage" else 0,
                              cond_channels=192 if shapes["kind"] == "zimage" else 0, seed=args.seed)
    sampler = torch.utils.data.distributed.DistributedSampler(ds, num_replicas=par.dp_size, rank=dp_rank,
                                                              shuffle=True, seed=args.seed)
    loader = torch.utils.data.DataLoader(ds, batch_size=args.train_batch_size, sampler=sampler, collate_fn=collate,
                                         num_workers=args.dataloader_num_workers, drop_last=True)

    global_step = 0
    if args.resume_from_checkpoint:
        path = latest_checkpoint(args.work_dir) if args.resume_from_checkpoint == "latest" else \
            args.resume_from_checkpoint
        if path:
            global_step = load_checkpoint(path, trainer, lrs)
            log.info(f"resumed from {path} at step {global_step}")
    trainer.opt.lr = lrs.lr()
    steps_per_epoch = max(1, len(loader))
    epochs = args.num_train_epochs or math.ceil(args.max_train_steps / steps_per_epoch)
    log.info(f"***** training {args.model}: world {world} sp {par.sp_size} dp {par.dp_size}, "
             f"{sum(p.numel() for p in model.parameters()) / 1e6:.1f}M params, {args.max_train_steps} steps *****")
    profiler = make_profiler(os.path.join(args.work_dir, "tb_profiler")) if args.enable_profiler else None
    if profiler:
        profiler.start()
    metrics = JsonlWriter(os.path.join(args.work_dir, "metrics.jsonl") if is_main else None)
    timer = PhaseTimer()
    img_tokens = None
    done = False
    skip = global_step % steps_per_epoch  # batches of the resumed epoch already trained on
    for epoch in range(global_step // steps_per_epoch, epochs):
        if done:
            break
        sampler.set_epoch(epoch)
        for batch in loader:
            if skip:
                skip -= 1
                continue
            fault.fire("step", global_step)
            t0 = time.time()
            latent = batch["latent_image"].to(torch.bfloat16)
            text = torch.stack(batch["prompt_embeds"]).to(torch.bfloat16)
            B = latent.shape[0]
            # per-(step, dp rank) generator: a resumed run draws the same noise and timesteps
            gen = torch.Generator().manual_seed((args.seed << 20) ^ (global_step << 8) ^ dp_rank)
            noise = torch.randn(latent.shape, generator=gen).to(torch.bfloat16)
            u = D.compute_density_for_timestep_sampling(args.weighting_scheme, B, args.logit_mean, args.logit_std,
                                                        args.mode_scale, generator=gen)
            idx = (u * sched.config.num_train_timesteps).long().clamp(max=sched.config.num_train_timesteps - 1)
            sigmas = sched.sigmas[idx]
            weighting = D.compute_loss_weighting_for_sd3(args.weighting_scheme, sigmas)
            host = {"latent": latent, "noise": noise, "text": text, "sigmas": sigmas, "weighting": weighting}
            if shapes["kind"] == "zimage":
                host["metadata"] = batch["norm_metadata"].to(torch.bfloat16)
                host["cond"] = [c.to(torch.bfloat16) for c in batch["cond"]]
            with timer.phase("step"):
                loss = trainer.step(host)
            lrs.step()
            trainer.opt.lr = lrs.lr()
            if use_cuda:
                errors.check(device)
            global_step += 1
            if img_tokens is None:
                p = 2
                img_tokens = (latent.shape[-1] // p) * (latent.shape[-2] // p)
            if global_step % args.log_interval == 0:
                ph = timer.report()
                rec = {"global_step": global_step, "step_loss": loss, "lr": lrs.lr(), "time": time.time() - t0,
                       "step_ms_max_over_ranks": ph.get("step"),
                       "image_tokens_per_s": (par.dp_size * B * img_tokens) / max(1e-9, ph.get("step", 0) / 1e3)}
                log.info(rec)
                metrics.write(rec)
            if profiler:
                profiler.step()
            if global_step % args.checkpointing_steps == 0:
                fault.fire("checkpoint", global_step)
                path = save_checkpoint(args.work_dir, global_step, trainer, lrs)
                log.info(f"saved {path}")
            if global_step >= args.max_train_steps:
                done = True
                break
        if done:
            break
    if profiler:
        profiler.stop()
        if is_main:
            print(profiler.key_averages().table(sort_by="self_cuda_time_total" if use_cuda else "self_cpu_time_total",
                                                row_limit=40))
    if use_cuda:
        torch.cuda.synchronize()
    trainer.close()  # a captured step (it may hold NCCL work) goes before the process group
    if world > 1:
        dist.barrier()
        from harp_b200.parallel.nvlink import NVLinkComm

        NVLinkComm.close_all()
        dist.destroy_process_group()
    return global_step


if __name__ == "__main__":
    main(parse_args())
