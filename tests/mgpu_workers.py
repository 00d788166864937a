"""Rank bodies for the multi-GPU tests (NCCL plus harp NVLink kernels, one
process per GPU).  Each writes <out>/rank<r>.pt."""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def entry(rank, world, port, name, out, args):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        res = globals()[name](rank, world, out, args)
        torch.save(res, os.path.join(out, f"rank{rank}.pt"))
    finally:
        from harp_b200.parallel.nvlink import NVLinkComm

        torch.cuda.synchronize()
        NVLinkComm.close_all()
        dist.destroy_process_group()


def train(rank, world, out, args):
    from harp_b200.models.dit import DiT, PRESETS
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    dev = torch.device("cuda", rank)
    model = DiT(PRESETS[args.get("model", "small")])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    par = ParallelState.build(world)
    tr = Trainer(model, par, TrainConfig(lr=1e-3, comm=args["comm"]), dev, sp_backend=args["backend"],
                 sp_mode=args["mode"])
    batch = torch.load(args["batch"])
    losses = [tr.step({k: v.pin_memory() for k, v in batch.items()}) for _ in range(args["steps"])]
    tr.check_errors()
    return {"losses": losses, "flat": tr.flat.flat.cpu(), "mode": tr.sp.mode, "backend": tr.sp.backend}


def flag_timeout(rank, world, out, args):
    """A flag that no peer ever sets: the bounded wait gives up after the
    timeout, records the error word and the context stays usable."""
    from harp_b200.parallel.nvlink import NVLinkComm, _BARRIER
    from harp_b200.runtime import errors

    dev = torch.device("cuda", rank)
    comm = NVLinkComm.get(dist.group.WORLD, dev)
    errors.word(dev).zero_()
    torch.ops.harp_comm.wait(comm.flags, _BARRIER, world, 1 << 30, 0.5, errors.word(dev))
    torch.cuda.synchronize(dev)
    e = errors.word(dev).cpu().tolist()
    x = (torch.ones(4, device=dev) * 2).sum().item()  # the context still works
    errors.word(dev).zero_()
    dist.barrier()
    return {"err": e, "x": x}
