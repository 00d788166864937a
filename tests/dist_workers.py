"""Rank bodies for the multi-process tests (gloo on CPU).  Each worker writes
its results to <out>/rank<r>.pt; the test process compares them."""
from __future__ import annotations

import datetime
import os
import sys
import time

import torch
import torch.distributed as dist


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    torch.manual_seed(1234)


def entry(rank, world, port, name, out, args):
    _init(rank, world, port, timeout_s=args.get("pg_timeout", 60) if isinstance(args, dict) else 60)
    try:
        res = globals()[name](rank, world, out, args)
        torch.save(res, os.path.join(out, f"rank{rank}.pt"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


# ---------------------------------------------------------------------------
def sp_attention(rank, world, out, args):
    from harp_b200.ops.modules import sp_attention as spa
    from harp_b200.parallel.sequence import SPContext

    B, S, H, Dh = 2, 32, 2, 16
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(B, S, H * Dh, generator=g).bfloat16() for _ in range(3))
    do = torch.randn(B, S, H * Dh, generator=g).bfloat16()
    sp = SPContext.from_group(dist.group.WORLD, backend="torch", mode=args.get("mode", "ring"))
    n = S // world
    sl = slice(rank * n, (rank + 1) * n)
    ql, kl, vl = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
    o = spa(ql, kl, vl, H, Dh, sp)
    o.backward(do[:, sl])
    return {"o": o.detach(), "dq": ql.grad, "dk": kl.grad, "dv": vl.grad, "sl": (sl.start, sl.stop),
            "q": q, "k": k, "v": v, "do": do}


def trainer_run(rank, world, out, args):
    from harp_b200.models.dit import DiT, PRESETS
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    sp_size = args["sp"]
    model = DiT(PRESETS["tiny"])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    par = ParallelState.build(sp_size)
    tr = Trainer(model, par, TrainConfig(lr=1e-3, weight_decay=0.01), "cpu", sp_mode=args.get("mode", "auto"))
    batch = torch.load(args["batch"])
    dp_rank = rank // sp_size
    per = batch["latent"].shape[0] // par.dp_size
    sel = slice(dp_rank * per, (dp_rank + 1) * per)
    losses = []
    for step in range(args["steps"]):
        b = {k: v[sel] for k, v in batch.items()}
        losses.append(tr.step(b))
    # parameters in registration order (independent of the flat buffer's bucket layout)
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    return {"losses": losses, "flat": flat, "sd": {k: v.clone() for k, v in model.state_dict().items()}}


def managers(rank, world, out, args):
    from harp_b200.managers.grad_manager import AsyncGradSyncManager
    from harp_b200.managers.shard_manager import SequenceAllGather, SequenceScatter, SPBroadcast
    from harp_b200.managers.weight_manager import (AsyncParamAllGatherManager, build_balanced_param_groups,
                                                   build_chunk_param, set_opt_hook)

    res = {}
    grp = dist.group.WORLD
    # sequence scatter / all-gather / broadcast
    x = torch.arange(2 * 8 * 3, dtype=torch.float32).view(2, 8, 3).requires_grad_(True)
    loc = SequenceScatter.apply(x, grp)
    res["scatter"] = loc.detach().clone()
    (loc * (rank + 1)).sum().backward()
    res["scatter_grad"] = x.grad.clone()
    y = torch.full((1, 2, 2), float(rank)).requires_grad_(True)
    full = SequenceAllGather.apply(y, grp)
    res["gather"] = full.detach().clone()
    (full * torch.arange(4.0).view(1, 4, 1)).sum().backward()
    res["gather_grad"] = y.grad.clone()
    z = torch.ones(3, requires_grad=True)
    (SPBroadcast.apply(z, grp) * (rank + 1)).sum().backward()
    res["bcast_grad"] = z.grad.clone()

    # balanced ownership + row chunks + background all-gather
    torch.manual_seed(5)
    model = torch.nn.Sequential(torch.nn.Linear(8, 8), torch.nn.LayerNorm(8), torch.nn.Linear(8, 4))
    mine, prank = build_balanced_param_groups(model, world, rank, block_size=100)
    res["owners"] = [prank[id(p)] for p in model.parameters()]
    for p in model.parameters():
        p.shared_grad = torch.zeros_like(p)
        p.state = torch.zeros((), dtype=torch.uint8)
    chunks = build_chunk_param(list(model.parameters()), model, world, rank)
    res["chunk_rows"] = [(getattr(c, "chunk_begin", 0), getattr(c, "chunk_end", c.shape[0] if c.ndim else 0))
                         for c in chunks]
    before = [p.detach().clone() for p in model.parameters()]
    hooks = set_opt_hook(model, timeout_s=30)
    mgr = AsyncParamAllGatherManager(grp, world)
    for p in model.parameters():
        if hasattr(p, "chunk_part"):
            p.chunk_part.data.add_(float(rank + 1))  # "optimizer step" on this rank's rows
            mgr.push(p)
    mgr.wait_all()
    model(torch.ones(1, 8))  # pre-hooks see every gathered parameter ready
    for h in hooks:
        h.remove()
    mgr.shutdown()
    res["gathered_delta"] = [(p.detach() - b) for p, b in zip(model.parameters(), before)]

    # gradient sync, three communication modes.  The RS group (rows of a
    # parameter) and the DP group (replicas) are orthogonal: mode 0 uses a
    # DP group of both ranks; modes 1/2 an RS group of both ranks and a DP group
    # of one.
    solo = [dist.new_group([r]) for r in range(world)][rank]
    for mode in (0, 1, 2):
        torch.manual_seed(9)
        m2 = torch.nn.Sequential(torch.nn.Linear(4, 4), torch.nn.Linear(4, 4))
        for p in m2.parameters():
            p.shared_grad = torch.zeros_like(p)
        params = list(m2.parameters())
        if mode:
            build_chunk_param(params, m2, world, rank)
        gm = AsyncGradSyncManager(m2, rank, 0, {id(p): rank for p in params}, set(params), sp_group=None,
                                  dp_group=grp if mode == 0 else solo, rs_group=grp, comm_mode=mode,
                                  replicated=lambda n: True)
        (m2(torch.full((2, 4), float(rank + 1))).sum()).backward()
        gm.wait_for_completion()
        gm.shutdown()
        res[f"grad_mode{mode}"] = [((p.chunk_part.grad.clone(), p.chunk_part.chunk_begin) if mode and
                                    hasattr(p, "chunk_part") else (p.shared_grad.clone(), 0)) for p in params]
    return res


def checkpoint(rank, world, out, args):
    from harp_b200.models.dit import DiT, PRESETS
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer
    from harp_b200.utils.checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
    from harp_b200.utils.diffusion import LRSchedule

    model = DiT(PRESETS["tiny"])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    tr = Trainer(model, ParallelState.build(world), TrainConfig(lr=1e-3), "cpu")
    lrs = LRSchedule("linear", 1e-3, num_warmup_steps=1, num_training_steps=10)
    batch = torch.load(args["batch"])
    tr.step(batch)
    lrs.step()
    save_checkpoint(args["dir"], 1, tr, lrs)
    snap = (tr.flat.flat.clone(), tr.opt.master.clone(), tr.opt.m.clone(), tr.opt.v.clone(), lrs.lr())
    tr.step(batch)  # move everything away from the snapshot
    lrs.step()
    path = latest_checkpoint(args["dir"])
    step = load_checkpoint(path, tr, lrs)
    now = (tr.flat.flat.clone(), tr.opt.master.clone(), tr.opt.m.clone(), tr.opt.v.clone(), lrs.lr())
    l2 = tr.step(batch)
    return {"step": step, "snap": snap, "now": now, "loss_after_resume": l2, "path": path}


def rank_exit(rank, world, out, args):
    """Rank 1 leaves between steps (nothing of its own in flight); rank 0 must
    see its next collective fail inside the process-group timeout."""
    from harp_b200.utils.fault import FaultInjector, Heartbeat

    os.environ["HARP_FAULT_RANK"] = "1"
    f = FaultInjector("exit@step:2", rank=rank)
    hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world, period_s=0.05)
    t = torch.ones(4)
    for step in range(4):
        f.fire("step", step)
        t0 = time.time()
        try:
            dist.all_reduce(t)
        except Exception as e:  # noqa: BLE001 - any transport error counts as detection
            time.sleep(0.5)
            stale = hb.stale(0.2)
            time.sleep(0.5)
            stale = hb.stale(0.2)
            hb.stop()
            return {"failed_at": step, "elapsed": time.time() - t0, "error": type(e).__name__, "stale": stale}
    hb.stop()
    return {"failed_at": None}


def groups(rank, world, out, args):
    from harp_b200.trainer import ParallelState

    par = ParallelState.build(args["sp"], args["rs"])
    get = lambda g: dist.get_process_group_ranks(g) if g is not None else None  # noqa: E731
    return {"sp": get(par.sp_group), "dp": get(par.dp_group), "rs": get(par.rs_group), "rs_size": par.rs_size}


def baseline_mmdit(rank, world, out, args):
    """The NCCL + cuBLAS/SDPA comparison arm's MMDiT trainer (replicated weights
    under DDP, or FSDP2 per-block sharding) on gloo: losses of a few steps."""
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline"))
    from mmdit_baseline import BaselineMMDiTTrainer

    tr = BaselineMMDiTTrainer(args["model"], torch.device("cpu"), world, shard=args.get("shard", False))
    b = torch.load(args["batch"])
    return {"losses": [float(tr.train_step(b["latent"], b["noise"], b["text"], b["sigmas"])) for _ in range(3)]}


class _HostComm:
    """Stand-in for the NVLink communicator's buffer API on CPU: plain tensors
    for the flat parameter/gradient buffers and the two staging slots."""

    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def allocate_flat(self, numel, param_numel=None):
        pn = numel if param_numel is None else param_numel
        return torch.zeros(pn, dtype=torch.bfloat16), torch.zeros(numel, dtype=torch.bfloat16)

    def param_slots(self, numel):
        self._slots = torch.zeros(2 * numel, dtype=torch.bfloat16)
        self._slot_numel = numel
        return self._slots

    def slot_view(self, s):
        return self._slots[s * self._slot_numel:(s + 1) * self._slot_numel]


def sharded_layout(rank, world, out, args):
    """ShardedFlatParams on gloo ranks with the host stand-in: each rank keeps
    1/world of every block bucket, the replicated rest sits at the start of the
    parameter buffer, and the gathered views reproduce the model."""
    from harp_b200.models.mmdit import MMDiT, PRESETS
    from harp_b200.parallel.param_shard import ShardedFlatParams, shard_groups

    torch.manual_seed(0)
    model = MMDiT(PRESETS["flux-tiny"])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    ref = {n: p.detach().clone() for n, p in model.named_parameters()}
    comm = _HostComm(rank, world)
    flat = ShardedFlatParams(model, torch.device("cpu"), comm, align=64)
    res = {"n_groups": len(shard_groups(model)), "rest": flat.rest_bucket, "buckets": len(flat.buckets)}
    views = flat.state_dict_views(dist.group.WORLD)
    res["views_match"] = all(torch.equal(views[n], ref[n]) for n in ref)
    # gather each block bucket by hand into slot 0 and point the block at it
    name_of = {id(p): n for n, p in zip(flat.names, flat.params)}
    ok = True
    for b in flat.bucket_params:
        lo, hi = flat.buckets[b]
        full = flat.full_bucket(b, dist.group.WORLD)
        comm.slot_view(0)[:hi - lo].copy_(full)
        flat.point(b, 0)
        for p, rel in flat.bucket_params[b]:
            ok = ok and torch.equal(p.data, ref[name_of[id(p)]])
        nb = (hi - lo) // world
        ok = ok and torch.equal(flat.local_slice(b), full[rank * nb:(rank + 1) * nb])
        ok = ok and flat.local_out(b) is not None
    res["points_match"] = ok
    res["rest_local"] = flat.local_out(flat.rest_bucket) is None
    return res


def _zimage_model():
    from harp_b200.models import zimage as Z

    torch.manual_seed(0)
    base = Z.ZImageTransformer2DModel(**Z.PRESETS["zimage-tiny"])
    model = Z.Z_Transformer(base, num_metadata=2, use_cond=True)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0, 0.05)
    return model.bfloat16()


def _zimage_batch(padded=False):
    """padded: an 18 x 18 latent (81 image tokens, padded to 96), a 20-token
    caption (padded to 32) and an 18 x 18 condition image, so pad tokens sit in
    the last rank's chunk of every run."""
    g = torch.Generator().manual_seed(8)
    hw, L = (18, 20) if padded else (16, 32)
    return {"lat": torch.randn(2, 16, hw, hw, generator=g).bfloat16(),
            "noise": torch.randn(2, 16, hw, hw, generator=g).bfloat16(),
            "text": torch.randn(2, L, 64, generator=g).bfloat16(), "sig": torch.rand(2, generator=g),
            "meta": torch.rand(2, 2, generator=g).bfloat16(),
            "cond": [torch.randn(2, 192, hw, hw, generator=g).bfloat16()]}


def zimage_sp(rank, world, out, args):
    """Z-Image SP wrapper (refiners, condition branch, metadata, joint layers)
    sequence-parallel over the gloo ranks: this rank's loss share and the
    gradients, summed over ranks by the caller."""
    from harp_b200.models import zimage as Z
    from harp_b200.parallel.sequence import SPContext

    model = _zimage_model()
    if args.get("ckpt"):
        model.gradient_checkpointing_enable()
    b = _zimage_batch(args.get("padded", False))
    sp = SPContext.from_group(dist.group.WORLD, backend="torch", mode=args.get("mode", "ring"))
    loss = Z.zimage_loss_local(model, b["lat"], b["noise"], b["text"], b["sig"], sp, metadata=b["meta"],
                               cond=b["cond"])
    loss.backward()
    grads = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1)
                       for p in model.parameters()])
    return {"loss": float(loss), "grads": grads}


def zimage_forward_full(rank, world, out, args):
    """The SP wrapper's forward (the reference's output contract: the full
    predictions on every rank) over the gloo ranks, with a loss computed in
    full on every rank as the reference's trainer does: the predictions and
    this rank's parameter gradients."""
    from harp_b200.models import zimage as Z
    from harp_b200.parallel.sequence import SPContext

    model = _zimage_model()
    b = _zimage_batch(args.get("padded", False))
    sp = SPContext.from_group(dist.group.WORLD, backend="torch") if world > 1 else SPContext()
    x = list(b["lat"].unsqueeze(2).unbind(0))
    pred = model(x, b["sig"], list(b["text"].unbind(0)), return_dict=False, metadata=b["meta"],
                 cond_list=b["cond"], sp=sp)[0]
    loss = sum((p.float() * (i + 1)).pow(2).mean() for i, p in enumerate(pred))
    loss.backward()
    grads = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1)
                       for p in model.parameters()])
    return {"pred": [p.detach().float() for p in pred], "grads": grads}


def _mmdit_setup(name):
    from harp_b200.models import mmdit as M

    torch.manual_seed(0)
    model = M.MMDiT(M.PRESETS[name])
    model.initialize_weights(0)
    with torch.no_grad():  # give the zero-initialised modulation and final layers some signal
        for n, p in model.named_parameters():
            if ".mod." in n or "adaLN" in n or "final_layer" in n:
                p.normal_(0, 0.02)
    model = model.bfloat16()
    cfg = M.PRESETS[name]
    g = torch.Generator().manual_seed(4)
    b = {"lat": torch.randn(1, cfg.in_channels, 16, 16, generator=g).bfloat16(),
         "noise": torch.randn(1, cfg.in_channels, 16, 16, generator=g).bfloat16(),
         "text": torch.randn(1, 32, cfg.text_dim, generator=g).bfloat16(), "sig": torch.rand(1, generator=g)}
    return model, b


def mmdit_sp(rank, world, out, args):
    """MMDiT / Flux sequence-parallel over the gloo ranks (the text stream
    lives on the last rank only): this rank's loss share and gradients."""
    from harp_b200.models import mmdit as M
    from harp_b200.parallel.sequence import SPContext

    model, b = _mmdit_setup(args["model"])
    sp = SPContext.from_group(dist.group.WORLD, backend="torch", mode=args.get("mode", "ring"))
    loss = M.mmdit_loss_local(model, b["lat"], b["noise"], b["text"], b["sig"], sp)
    loss.backward()
    grads = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1)
                       for p in model.parameters()])
    return {"loss": float(loss), "grads": grads}


def ring_ops_sp(rank, world, out, args):
    """The reference's ring_attention_ops (through CPURingAttention) over the
    gloo ranks: each rank's chunk of the output and of dQ/dK/dV."""
    from harp_b200.ops import ring_ops
    from harp_b200.parallel.sequence import SPContext

    g = torch.Generator().manual_seed(21)
    B, H, T, D = 1, 2, 24 * world, 32
    q, k, v, do = (torch.randn(B, H, T, D, generator=g).bfloat16() for _ in range(4))
    t = T // world
    sl = slice(rank * t, (rank + 1) * t)
    # token-major storage viewed as [B, H, T_local, D], as the reference passes it
    ql, kl, vl = (x[:, :, sl].transpose(1, 2).contiguous().transpose(1, 2).requires_grad_(True) for x in (q, k, v))
    ring_ops.set_sp_context(SPContext.from_group(dist.group.WORLD, backend="torch", mode="ring"))
    o = ring_ops.CPURingAttention.apply(ql, kl, vl, world)
    o.backward(do[:, :, sl])
    ring_ops.set_sp_context(None)
    return {"o": o.detach().float(), "dq": ql.grad.float(), "dk": kl.grad.float(), "dv": vl.grad.float()}


def _load_reference(ref_dir, rel):
    import importlib.util

    spec = importlib.util.spec_from_file_location("_reference_" + rel.replace("/", "_")[:-3],
                                                  os.path.join(ref_dir, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _IdentityList(list):
    def __contains__(self, x):
        return any(x is y for y in self)


class _GlooAllGatherShape:
    """torch.distributed, except that all_gather_into_tensor passes its output
    to the backend as the inputs concatenated along dim 0 (the same memory as
    the [world, *input] stacked form the reference allocates).  NCCL takes
    either shape; gloo takes only the concatenated one."""

    def __getattr__(self, name):
        return getattr(dist, name)

    @staticmethod
    def all_gather_into_tensor(output, inp, group=None, async_op=False):
        return dist.all_gather_into_tensor(output.view(-1, *inp.shape[1:]), inp, group=group, async_op=async_op)


def managers_oracle(rank, world, out, args):
    """The reference's managers/shard_manager.py and the pure-PyTorch parts of
    managers/weight_manager.py, run beside harp's on the same inputs over the
    gloo ranks: sequence scatter / all-gather / broadcast (forward and
    backward), byte-balanced ownership, row chunks and the background
    all-gather of updated chunks."""
    from harp_b200.managers import shard_manager as HS
    from harp_b200.managers import weight_manager as HW

    RS = _load_reference(args["ref"], "managers/shard_manager.py")
    RW = _load_reference(args["ref"], "managers/weight_manager.py")
    RS.dist = _GlooAllGatherShape()
    grp = dist.group.WORLD
    res = {}
    for B in (1, 3):
        g = torch.Generator().manual_seed(11 + B)
        full = torch.randn(B, 4 * world, 5, generator=g)
        loc = torch.randn(B, 4, 5, generator=g) + rank
        w_full = torch.randn(B, 4 * world, 5, generator=g)
        w_loc = torch.randn(B, 4, 5, generator=g)
        for tag, mod in (("ref", RS), ("ours", HS)):
            x = full.clone().requires_grad_(True)
            y = mod.SequenceScatter.apply(x, grp)
            (y * w_loc * (rank + 1)).sum().backward()
            res[f"scatter{B}_{tag}"] = (y.detach(), x.grad)
            x = loc.clone().requires_grad_(True)
            y = mod.SequenceAllGather.apply(x, grp)
            (y * w_full).sum().backward()
            res[f"gather{B}_{tag}"] = (y.detach(), x.grad)
            x = loc.clone().requires_grad_(True)
            (mod.SPBroadcast.apply(x, grp) * (rank + 2)).sum().backward()
            res[f"bcast{B}_{tag}"] = x.grad

    def make_model():
        torch.manual_seed(5)
        return torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.LayerNorm(16), torch.nn.Linear(16, 8),
                                   torch.nn.RMSNorm(8), torch.nn.Linear(8, 4))

    for tag, mod in (("ref", RW), ("ours", HW)):
        model = make_model()
        params = list(model.parameters())
        idx = {id(p): i for i, p in enumerate(params)}
        mine, prank = mod.build_balanced_param_groups(model, world, rank, block_size=200)
        res[f"owners_{tag}"] = [prank.get(id(p)) for p in params]
        res[f"mine_{tag}"] = [idx[id(p)] for p in mine]
        for p in params:
            p.shared_grad = torch.arange(p.numel(), dtype=p.dtype).view(p.shape) + idx[id(p)]
            p.state = torch.zeros((), dtype=torch.uint8)
        # row chunks over an RS group of both ranks: its members optimize the
        # same parameters (an owner's), here all of them.  The reference tests
        # `p in my_params`, which compares tensors by value and raises once two
        # parameters of different shapes meet; it means identity, which is
        # what this list's membership test does
        owned = _IdentityList(p for p in params if p.requires_grad)
        chunks = mod.build_chunk_param(owned, model, world, rank)
        res[f"chunks_{tag}"] = [(getattr(c, "chunk_begin", None), getattr(c, "chunk_end", None), c.detach().clone(),
                                 None if c.grad is None else c.grad.clone()) for c in chunks]
        mgr = mod.AsyncParamAllGatherManager(grp, world)
        for p in params:
            if hasattr(p, "chunk_part"):
                p.chunk_part.data.mul_(float(rank + 2))  # this rank's "optimizer step" on its rows
                mgr.push(p)
        mgr.wait_all()
        mgr.shutdown()
        res[f"params_{tag}"] = [p.detach().clone() for p in params]
        res[f"state_{tag}"] = [int(p.state) for p in params]
    return res


def zimage_reference_sp(rank, world, out, args):
    """The reference's own sequence-parallel Z-Image (src/models/z_image/
    hl_model.py with its module/block.py and module/attn.py, on its
    standalone base model) beside harp's Z_Transformer(harp_block_compat=True)
    with the same weights.  The reference's imports of managers.*, async_rt.*
    and its ring-attention ops resolve to this repository's implementations of
    those APIs (harp_b200.compat registers the module names before the
    reference's directory joins sys.path).

    The reference runs on a one-rank group, in fp32 and in bf16, so its
    gradients are the exact ones: over several ranks it all-reduces the adaLN
    input's gradient once per section (SPBroadcast), summing gradients that are
    already sums, so t_embedder and the metadata embedders come out inflated.
    Over the whole group it runs the forward only, in bf16.
    harp runs sequence-parallel over the whole group in bf16.  Returns the
    image predictions (the reference's in full, harp's for this rank's tokens)
    and the parameter gradients of a fixed weighted sum of the predictions."""
    import sys

    from harp_b200.compat import install_reference_import_paths

    install_reference_import_paths()
    sys.path.append(args["ref"])
    from src.models.z_image import hl_model as RH
    from src.models.z_image import standalone_transformer as RS

    from harp_b200.models import zimage as Z
    from harp_b200.ops import ring_ops
    from harp_b200.parallel.sequence import SPContext

    grp = dist.group.WORLD
    solo = [dist.new_group([r]) for r in range(world)][rank]
    sp = SPContext.from_group(grp, backend="torch") if world > 1 else SPContext()
    pre = dict(Z.PRESETS["zimage-tiny"])

    def reference_model(group, size):
        torch.manual_seed(0)
        base = RS.ZImageTransformer2DModel(**{k: (list(v) if isinstance(v, tuple) else v) for k, v in pre.items()})
        return RH.Z_Transformer(base, num_metadata=2, use_cond=True, sp_group_model=group, sp_size=size)

    ref32 = reference_model(solo, 1)
    with torch.no_grad():
        for p in ref32.parameters():
            p.normal_(0, 0.05)
    ref16 = reference_model(solo, 1)
    ref16.load_state_dict(ref32.state_dict(), strict=True)
    obase = Z.ZImageTransformer2DModel(**pre)
    ours = Z.Z_Transformer(obase, num_metadata=2, use_cond=True, sp_size=world, harp_block_compat=True)
    ours.load_state_dict(ref32.state_dict(), strict=True)
    ref32, ref16, ours = ref32.float(), ref16.bfloat16(), ours.bfloat16()

    g = torch.Generator().manual_seed(3)
    B, hw = 2, args.get("hw", 16)
    x = [torch.randn(16, 1, hw, hw, generator=g).bfloat16() for _ in range(B)]
    t = torch.rand(B, generator=g)
    caps = [torch.randn(args.get("cap", 32), pre["cap_feat_dim"], generator=g).bfloat16() for _ in range(B)]
    meta = torch.rand(B, 2, generator=g).bfloat16()
    cond = [[torch.randn(192, hw, hw, generator=g).bfloat16() for _ in range(B)]]
    n_img = (hw // 2) ** 2
    w = torch.randn(B, n_img, 4 * 16, generator=g)

    def grads(m):
        return {n: (p.grad.float().clone() if p.grad is not None else torch.zeros(p.shape)) for n, p in
                m.named_parameters()}

    def run_reference(m, dt):
        pred = m([v.to(dt) for v in x], t, [c.to(dt) for c in caps], metadata=meta.to(dt),
                 cond_list=[[c.to(dt) for c in branch] for branch in cond]).sample
        return torch.stack(obase.patchify([p.float() for p in pred], 2, 1)[0])  # [B, n_img, p*p*C]

    res = {}
    ring_ops.set_sp_context(None)
    for tag, m, dt in (("ref32", ref32, torch.float32), ("ref16", ref16, torch.bfloat16)):
        tok = run_reference(m, dt)
        (tok * w).sum().backward()
        res["pred_" + tag], res["grads_" + tag] = tok.detach(), grads(m)
    if world > 1:
        refw = reference_model(grp, world)
        refw.load_state_dict(ref32.state_dict(), strict=True)
        ring_ops.set_sp_context(sp)
        with torch.no_grad():
            res["pred_refw"] = run_reference(refw.bfloat16(), torch.bfloat16)
    pred_o, lo, hi = ours.forward_local(x, t, caps, metadata=meta, cond_list=cond, sp=sp)
    (pred_o.float() * w[:, lo:hi]).sum().backward()
    res.update(pred_ours=pred_o.detach().float(), range=(lo, hi), grads_ours=grads(ours))
    return res
