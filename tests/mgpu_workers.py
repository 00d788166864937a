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
    cfg = TrainConfig(lr=1e-3, comm=args["comm"], overlap_grad_sync=args.get("overlap", True),
                      bucket_params=args.get("bucket_params", 64_000_000), shard_params=args.get("shard", False),
                      cuda_graph=args.get("graph", False), graph_warmup=2)
    tr = Trainer(model, par, cfg, dev, sp_backend=args["backend"], sp_mode=args["mode"])
    batch = torch.load(args["batch"])
    losses = [tr.step({k: v.pin_memory() for k, v in batch.items()}) for _ in range(args["steps"])]
    tr.check_errors()
    graph_replays = tr._replays
    tr.close()
    # parameters in registration order (independent of the flat buffer's bucket
    # layout; with sharded parameters gathered from their owners)
    sd = tr.model_state_dict()
    flat = torch.cat([sd[n].detach().reshape(-1) for n, _ in model.named_parameters()]).cpu()
    return {"losses": losses, "flat": flat, "mode": tr.sp.mode, "backend": tr.sp.backend,
            "buckets": len(tr.flat.buckets), "overlap": tr._overlap, "graph_replays": graph_replays}


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


def c10d_backend(rank, world, out, args):
    """Every collective of the harp_nvl backend against values computed locally."""
    from harp_b200.parallel import c10d_backend as CB

    CB.register()
    g = dist.new_group(backend=CB.NAME)
    dev = torch.device("cuda", rank)
    res = {}
    for dtype in (torch.float32, torch.bfloat16):
        for n in (1000, 3_000_001):  # one-shot and two-phase all-reduce (odd length included)
            x = torch.arange(n, device=dev, dtype=torch.float32).to(dtype) * (rank + 1)
            dist.all_reduce(x, group=g)
            ref = torch.arange(n, device=dev, dtype=torch.float32).to(dtype).float() * sum(r + 1 for r in range(world))
            res[f"ar_{dtype}_{n}"] = (x.float() - ref).abs().max().item() / max(1.0, ref.abs().max().item())
    m = torch.tensor([float(rank)], device=dev)
    dist.all_reduce(m, op=dist.ReduceOp.MAX, group=g)
    res["max"] = m.item()
    x = torch.full((1025,), float(rank), device=dev)
    full = torch.empty(world * 1025, device=dev)
    dist.all_gather_into_tensor(full, x, group=g)
    res["ag"] = bool(torch.equal(full, torch.arange(world, device=dev).float().repeat_interleave(1025)))
    lst = [torch.empty(3, device=dev) for _ in range(world)]
    dist.all_gather(lst, torch.full((3,), rank + 0.5, device=dev), group=g)
    res["ag_list"] = [t.tolist() for t in lst]
    inp = torch.arange(world * 8, device=dev, dtype=torch.float32) + rank
    o = torch.empty(8, device=dev)
    dist.reduce_scatter_tensor(o, inp, group=g)
    res["rs"] = bool(torch.equal(o, (torch.arange(world * 8, device=dev).float() * world
                                     + sum(range(world)))[rank * 8:(rank + 1) * 8]))
    b = torch.full((77,), float(rank), device=dev)
    dist.broadcast(b, src=world - 1, group=g)
    res["bcast"] = bool(torch.all(b == world - 1))
    a_in = torch.arange(world * 4, device=dev, dtype=torch.float32) + 100 * rank
    a_out = torch.empty_like(a_in)
    dist.all_to_all_single(a_out, a_in, group=g)
    exp = torch.cat([torch.arange(rank * 4, rank * 4 + 4, device=dev).float() + 100 * r for r in range(world)])
    res["a2a"] = bool(torch.equal(a_out, exp))
    dist.barrier(group=g)
    w = dist.all_reduce(torch.ones(4, device=dev), group=g, async_op=True)
    w.wait()
    torch.cuda.synchronize()
    res["async"] = True
    dist.destroy_process_group(g)
    return res


def nvl_world1(rank, world, out, args):
    """The NVLink exchange kernels on a one-rank group (every peer pointer is
    this GPU's own buffer): fused Ulysses dispatch / remaps and the ring K/V
    dispatch + dK/dV push, through attention forward and backward, against
    fp32 SDPA.  Returns max errors relative to each reference's largest value."""
    import torch.nn.functional as F

    from harp_b200.parallel.nvlink import NVLinkComm
    from harp_b200.runtime import errors

    dev = torch.device("cuda", rank)
    comm = NVLinkComm.get(dist.group.WORLD, dev)
    B, S, H, Dh = 2, 384, 2, 64
    g = torch.Generator(device=dev).manual_seed(11)
    qkv = torch.randn(B * S, 3 * H * Dh, device=dev, generator=g).bfloat16()
    do = torch.randn(B * S, H * Dh, device=dev, generator=g).bfloat16()

    def heads(x):
        return x.float().reshape(B, S, H, Dh).transpose(1, 2)

    def rows(x):
        return x.transpose(1, 2).reshape(B * S, H * Dh)

    q, k, v = (heads(t).requires_grad_(True) for t in qkv.split(H * Dh, 1))
    ref = F.scaled_dot_product_attention(q, k, v)
    ref.backward(heads(do))
    ref_o = rows(ref.detach())
    ref_d = [rows(t.grad) for t in (q, k, v)]

    def rel(a, b):
        return ((a.float() - b).abs().max() / b.abs().max()).item()

    res = {}
    comm.begin_step()
    o, _, _, saved = comm.uly_forward(qkv, B, S, H, Dh, None, None, None, 0.0, False)
    dqkv = comm.uly_backward(saved, do, B, S, H, Dh)
    torch.cuda.synchronize()
    res["uly_o"] = rel(o, ref_o)
    res["uly_dq"], res["uly_dk"], res["uly_dv"] = (rel(t, r) for t, r in zip(dqkv.split(H * Dh, 1), ref_d))
    comm.begin_step()
    qs, ks, vs = (t.contiguous() for t in qkv.split(H * Dh, 1))
    o2, q2, _, _, saved2 = comm.ring_forward(qs, ks, vs, B, S, H, Dh, q_ready=True)
    dq2, dkv2 = comm.ring_backward(saved2, q2, o2, do, B, S, H, Dh)
    torch.cuda.synchronize()
    res["ring_o"] = rel(o2, ref_o)
    res["ring_dq"] = rel(dq2, ref_d[0])
    res["ring_dk"], res["ring_dv"] = (rel(t, r) for t, r in zip(dkv2.split(H * Dh, 1), ref_d[1:]))
    errors.check(dev)
    return res
