"""Checkpoint / resume (reference: train.py:302-329 resume, :556-566 save).

Layout of `<work_dir>/checkpoint-<step>/` (the reference's file names kept):
  pytorch_model.bin        full model state_dict (bf16), written by rank 0
  optimizer.rank<k>.bin    rank k's optimizer shard (fp32 master, exp_avg,
                           exp_avg_sq, step) - every rank writes its own
  optimizer.bin            consolidated optimizer state (consolidate=True)
  scheduler.bin            LR-schedule state, rank 0
  meta.json                step, world size, flat-buffer layout
The reference saves only rank 0's optimizer chunk and no weights, and its
resume path references objects before they exist (see its train.py:324-329);
here every rank's shard is saved and resume restores weights, optimizer
shards and the schedule, bit-exactly.
"""
from __future__ import annotations

import json
import os
import re
from typing import Optional

import torch
import torch.distributed as dist


def _barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def checkpoint_dir(work_dir: str, step: int) -> str:
    return os.path.join(work_dir, f"checkpoint-{step}")


def latest_checkpoint(work_dir: str) -> Optional[str]:
    """Newest complete checkpoint-<step> under `work_dir` or one level below it
    (train.py puts each run in a timestamped sub-directory)."""
    if not os.path.isdir(work_dir):
        return None
    best, path = (-1, 0.0), None
    roots = [work_dir] + [os.path.join(work_dir, d) for d in os.listdir(work_dir)
                          if os.path.isdir(os.path.join(work_dir, d))]
    for root in roots:
        for d in os.listdir(root):
            m = re.fullmatch(r"checkpoint-(\d+)", d)
            meta = os.path.join(root, d, "meta.json")
            if m and os.path.exists(meta):
                key = (int(m.group(1)), os.path.getmtime(meta))
                if key > best:
                    best, path = key, os.path.join(root, d)
    return path


def save_checkpoint(work_dir: str, step: int, trainer, schedule=None, consolidate: bool = False) -> str:
    rank = trainer.par.rank
    world = trainer.par.world_size
    path = checkpoint_dir(work_dir, step)
    if rank == 0:
        os.makedirs(path, exist_ok=True)
    _barrier()
    torch.cuda.synchronize() if torch.cuda.is_available() else None
    # every rank takes part: with sharded parameters this gathers the weights
    full = trainer.model_state_dict() if hasattr(trainer, "model_state_dict") else trainer.model.state_dict()
    if rank == 0:
        sd = {k: v.detach().cpu() for k, v in full.items()}
        torch.save(sd, os.path.join(path, "pytorch_model.bin"))
        if schedule is not None:
            torch.save(schedule.state_dict(), os.path.join(path, "scheduler.bin"))
    torch.save(trainer.opt.state_dict(), os.path.join(path, f"optimizer.rank{rank}.bin"))
    _barrier()
    if consolidate and rank == 0:
        shards = [torch.load(os.path.join(path, f"optimizer.rank{r}.bin")) for r in range(world)]
        full = {k: torch.cat([s[k] for s in shards]) for k in ("master", "exp_avg", "exp_avg_sq")}
        full.update(step=shards[0]["step"], lr=shards[0]["lr"], world=world)
        torch.save(full, os.path.join(path, "optimizer.bin"))
    if rank == 0:
        meta = {"step": step, "world": world, "flat_numel": trainer.flat.numel, "names": trainer.flat.names,
                "offsets": trainer.flat.offsets}
        with open(os.path.join(path, "meta.json"), "w") as fh:
            json.dump(meta, fh)
    _barrier()
    return path


def load_checkpoint(path: str, trainer, schedule=None) -> int:
    """Restore a checkpoint written by save_checkpoint (same world size)."""
    with open(os.path.join(path, "meta.json")) as fh:
        meta = json.load(fh)
    if meta["world"] != trainer.par.world_size:
        raise ValueError(f"checkpoint written by {meta['world']} ranks, running {trainer.par.world_size}")
    sd = torch.load(os.path.join(path, "pytorch_model.bin"), map_location="cpu")
    missing, unexpected = trainer.model.load_state_dict(sd, strict=False)
    if missing or unexpected:
        raise KeyError(f"state_dict mismatch: missing {missing[:5]} unexpected {unexpected[:5]}")
    opt_sd = torch.load(os.path.join(path, f"optimizer.rank{trainer.par.rank}.bin"), map_location="cpu")
    trainer.opt.load_state_dict(opt_sd)
    if schedule is not None and os.path.exists(os.path.join(path, "scheduler.bin")):
        schedule.load_state_dict(torch.load(os.path.join(path, "scheduler.bin")))
    trainer.global_step = meta["step"]
    return meta["step"]
