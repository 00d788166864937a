"""Multi-process tests on CPU (gloo, 2 and 4 ranks): sequence-parallel
attention, trainer parity (SP and DP against one process), the managers API,
the model families under sequence parallelism, sharded checkpoints, detection
of a rank that leaves, and (with HARP_REFERENCE_DIR) the reference's own
managers and SP Z-Image beside harp's.  Multi-rank paths are checked against
a single-rank run of the same math."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

import dist_workers as W

pytestmark = pytest.mark.timeout(600)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(name, world, tmp_path, args=None, expect_ok=True):
    ctx = mp.get_context("spawn")
    port = _port()
    out = str(tmp_path)
    procs = [ctx.Process(target=W.entry, args=(r, world, port, name, out, args or {})) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    if expect_ok:
        assert codes == [0] * world, codes
    res = {}
    for r in range(world):
        f = os.path.join(out, f"rank{r}.pt")
        if os.path.exists(f):
            res[r] = torch.load(f, weights_only=False)
    return res, codes


def _full_attention(q, k, v, do, H, Dh):
    q, k, v = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    B, S, _ = q.shape
    qh, kh, vh = (t.view(B, S, H, Dh).transpose(1, 2) for t in (q, k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(B, S, H * Dh)
    o.backward(do.float())
    return o.detach(), q.grad, k.grad, v.grad


@pytest.mark.parametrize("mode", ["ring", "ulysses"])
def test_sp_attention_two_ranks_matches_full(tmp_path, mode):
    res, _ = _run("sp_attention", 2, tmp_path, {"mode": mode})
    r0 = res[0]
    o, dq, dk, dv = _full_attention(r0["q"], r0["k"], r0["v"], r0["do"], 2, 16)
    for r in (0, 1):
        lo, hi = res[r]["sl"]
        for key, ref in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
            got = res[r][key].float()
            want = ref[:, lo:hi]
            err = ((got - want).norm() / want.norm()).item()
            assert err < 2e-2, (r, key, err)


def _batch(path, n=2, seed=3):
    from harp_b200.models.dit import PRESETS

    cfg = PRESETS["tiny"]
    g = torch.Generator().manual_seed(seed)
    b = {"latent": torch.randn(n, cfg.in_channels, 16, 16, generator=g).bfloat16(),
         "noise": torch.randn(n, cfg.in_channels, 16, 16, generator=g).bfloat16(),
         "text": torch.randn(n, 16, cfg.text_dim, generator=g).bfloat16(),
         "sigmas": torch.rand(n, generator=g)}
    torch.save(b, path)
    return b


def _single_run(batch, steps):
    from harp_b200.models.dit import DiT, PRESETS
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    torch.manual_seed(1234)
    model = DiT(PRESETS["tiny"])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    tr = Trainer(model, ParallelState(), TrainConfig(lr=1e-3, weight_decay=0.01), "cpu")
    losses = [tr.step(batch) for _ in range(steps)]
    return losses, torch.cat([p.detach().reshape(-1) for p in model.parameters()])


@pytest.mark.parametrize("sp,mode", [(2, "ring"), (2, "ulysses"), (1, "auto")])
def test_trainer_two_ranks_matches_single_process(tmp_path, sp, mode):
    bpath = str(tmp_path / "batch.pt")
    batch = _batch(bpath)
    ref_losses, ref_flat = _single_run(batch, 3)
    res, _ = _run("trainer_run", 2, tmp_path, {"sp": sp, "batch": bpath, "steps": 3, "mode": mode})
    for r in (0, 1):
        got = res[r]["losses"]
        assert got == pytest.approx(ref_losses, rel=2e-3), (r, got, ref_losses)
        # every rank holds the same (all-gathered) parameters as the single run,
        # up to one bf16 rounding step: gradients are summed in another order, and
        # where a gradient is ~0 AdamW's normalised step can flip sign (<= 2 lr a step)
        torch.testing.assert_close(res[r]["flat"].float(), ref_flat.float(), rtol=2 ** -7, atol=2 * 3 * 1e-3)
    assert torch.equal(res[0]["flat"], res[1]["flat"])


def test_managers_two_ranks(tmp_path):
    res, _ = _run("managers", 2, tmp_path)
    x = torch.arange(2 * 8 * 3, dtype=torch.float32).view(2, 8, 3)
    for r in (0, 1):
        d = res[r]
        torch.testing.assert_close(d["scatter"], x[:, r * 4:(r + 1) * 4])
        g = torch.zeros_like(x)
        g[:, 0:4] = 1.0
        g[:, 4:8] = 2.0
        torch.testing.assert_close(d["scatter_grad"], g)  # backward all-gathers every rank's chunk grad
        torch.testing.assert_close(d["gather"], torch.tensor([0., 0., 1., 1.]).view(1, 4, 1).expand(1, 4, 2))
        torch.testing.assert_close(d["gather_grad"], torch.arange(4.0)[r * 2:(r + 1) * 2].view(1, 2, 1).expand(1, 2, 2))
        torch.testing.assert_close(d["bcast_grad"], torch.full((3,), 3.0))  # 1 + 2 summed over SP
        assert d["owners"] == res[0]["owners"]
        # each rank added (rank+1) to its own rows; after the gather every rank sees both
        for delta, (b, e) in zip(d["gathered_delta"], res[0]["chunk_rows"]):
            if delta.ndim and delta.shape[0] % 2 == 0:
                h = delta.shape[0] // 2
                torch.testing.assert_close(delta[:h], torch.ones_like(delta[:h]))
                torch.testing.assert_close(delta[h:], torch.full_like(delta[h:], 2.0))
    # gradient modes: mode 0 holds the full summed gradient; modes 1/2 this rank's
    # rows of it; the union over ranks equals mode 0
    for r in (0, 1):
        for (g0, _), (g1, b1), (g2, b2) in zip(res[r]["grad_mode0"], res[r]["grad_mode1"], res[r]["grad_mode2"]):
            torch.testing.assert_close(g1, g0[b1:b1 + g1.shape[0]])
            torch.testing.assert_close(g2, g0[b2:b2 + g2.shape[0]])
    torch.testing.assert_close(res[0]["grad_mode0"][0][0], res[1]["grad_mode0"][0][0])


def test_sharded_checkpoint_roundtrip_two_ranks(tmp_path):
    bpath = str(tmp_path / "batch.pt")
    _batch(bpath)
    res, _ = _run("checkpoint", 2, tmp_path, {"batch": bpath, "dir": str(tmp_path / "ckpt")})
    for r in (0, 1):
        d = res[r]
        assert d["step"] == 1 and d["path"].endswith("checkpoint-1")
        for a, b in zip(d["snap"][:4], d["now"][:4]):
            assert torch.equal(a, b)  # bit-exact weights, master, moments
        assert d["snap"][4] == d["now"][4]
    assert os.path.exists(tmp_path / "ckpt" / "checkpoint-1" / "optimizer.rank1.bin")
    assert res[0]["loss_after_resume"] == res[1]["loss_after_resume"]


def test_rank_that_leaves_is_detected(tmp_path):
    res, codes = _run("rank_exit", 2, tmp_path, {"pg_timeout": 15}, expect_ok=False)
    assert codes[1] == 17  # the injected exit
    d = res[0]
    assert d["failed_at"] == 2, d
    assert d["elapsed"] < 30
    assert d["stale"] == [1], d


def test_group_topology_four_ranks(tmp_path):
    res, _ = _run("groups", 4, tmp_path, {"sp": 2, "rs": 2})
    # SP groups of consecutive ranks, DP groups of equal SP index, RS groups of
    # equal SP index inside blocks of sp*rs ranks
    assert [res[r]["sp"] for r in range(4)] == [[0, 1], [0, 1], [2, 3], [2, 3]]
    assert [res[r]["dp"] for r in range(4)] == [[0, 2], [1, 3], [0, 2], [1, 3]]
    assert [res[r]["rs"] for r in range(4)] == [[0, 2], [1, 3], [0, 2], [1, 3]]
    assert res[0]["rs_size"] == 2


@pytest.mark.parametrize("shard", [False, True])
def test_baseline_mmdit_two_ranks_matches_one(tmp_path, shard):
    """The comparison arm's MMDiT step, sequence-parallel over two gloo ranks
    (K/V all-gathered, DDP or FSDP2 gradients), follows the one-process run:
    the ranks' gradients are averaged instead of summed, which AdamW's update
    does not see beyond its epsilon."""
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline"))
    from mmdit_baseline import BaselineMMDiTTrainer

    g = torch.Generator().manual_seed(5)
    b = {"latent": torch.randn(1, 16, 16, 16, generator=g).bfloat16(),
         "noise": torch.randn(1, 16, 16, 16, generator=g).bfloat16(),
         "text": torch.randn(1, 32, 128, generator=g).bfloat16(), "sigmas": torch.rand(1, generator=g)}
    path = str(tmp_path / "batch.pt")
    torch.save(b, path)
    torch.manual_seed(0)
    one = BaselineMMDiTTrainer("flux-tiny", torch.device("cpu"), 1)
    ref = [float(one.train_step(b["latent"], b["noise"], b["text"], b["sigmas"])) for _ in range(3)]
    res, _ = _run("baseline_mmdit", 2, tmp_path, {"model": "flux-tiny", "batch": path, "shard": shard})
    for r in (0, 1):
        assert res[r]["losses"] == pytest.approx(ref, rel=2e-2), (res[r]["losses"], ref)


@pytest.mark.parametrize("sp,mode", [(4, "ring"), (2, "ring"), (2, "ulysses")])
def test_trainer_four_ranks_matches_single_process(tmp_path, sp, mode):
    """Parity above two ranks: sequence parallel over 4 ranks (K/V gather; the
    tiny model's 6 heads do not split 4 ways), and 2-way SP (K/V gather or head
    all-to-all) x 2-way DP, against the one-process run."""
    bpath = str(tmp_path / "batch.pt")
    batch = _batch(bpath)
    ref_losses, ref_flat = _single_run(batch, 3)
    res, _ = _run("trainer_run", 4, tmp_path, {"sp": sp, "batch": bpath, "steps": 3, "mode": mode})
    for r in range(4):
        assert res[r]["losses"] == pytest.approx(ref_losses, rel=2e-3), (r, res[r]["losses"], ref_losses)
        torch.testing.assert_close(res[r]["flat"].float(), ref_flat.float(), rtol=2 ** -7, atol=2 * 3 * 1e-3)
    for r in range(1, 4):
        assert torch.equal(res[0]["flat"], res[r]["flat"])


def test_sharded_weight_layout_two_ranks(tmp_path):
    """Host-side logic of sharded block weights (parallel/param_shard.py) on
    two gloo ranks with a CPU stand-in for the symmetric buffers: one bucket
    per block, each rank's slice, the gathered views and the staging-slot
    re-pointing all reproduce the model's parameters."""
    res, _ = _run("sharded_layout", 2, tmp_path)
    for r in (0, 1):
        assert res[r]["views_match"] and res[r]["points_match"] and res[r]["rest_local"], res[r]
        assert res[r]["buckets"] == res[r]["n_groups"] + 1 and res[r]["rest"] == res[r]["n_groups"], res[r]


@pytest.mark.parametrize("padded,world,mode", [(False, 2, "ring"), (True, 2, "ring"), (True, 4, "ring"),
                                               (True, 4, "ulysses")])
def test_zimage_two_ranks_match_one(padded, world, mode):
    """The Z-Image SP wrapper over two or four gloo ranks: the ranks' loss
    shares and gradients sum to the one-process loss and gradients (the
    reference never checks its SP model against a single-rank run); also with
    image, caption and condition runs that need pad tokens, whose padding then
    lands in the last ranks' chunks."""
    import tempfile

    from harp_b200.models import zimage as Z
    from harp_b200.parallel.sequence import SPContext

    model = W._zimage_model()
    b = W._zimage_batch(padded)
    loss = Z.zimage_loss_local(model, b["lat"], b["noise"], b["text"], b["sig"], SPContext(), metadata=b["meta"],
                               cond=b["cond"])
    loss.backward()
    ref_g = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1)
                       for p in model.parameters()])
    with tempfile.TemporaryDirectory() as d:
        res, _ = _run("zimage_sp", world, d, {"padded": padded, "mode": mode})
    tot = sum(res[r]["loss"] for r in range(world))
    assert tot == pytest.approx(float(loss), rel=2e-2), (tot, float(loss))
    g = sum(res[r]["grads"] for r in range(world))
    rel = ((g - ref_g).norm() / ref_g.norm()).item()
    assert rel < 2e-2, rel


@pytest.mark.parametrize("name,mode", [("flux-tiny", "ring"), ("mmdit-tiny", "ulysses")])
def test_mmdit_two_ranks_match_one(name, mode):
    """MMDiT / Flux (double- and single-stream blocks) over two gloo ranks: the
    loss shares and gradients sum to the one-process ones, including the text
    stream's weights, which only the rank holding text tokens uses."""
    import tempfile

    from harp_b200.models import mmdit as M
    from harp_b200.parallel.sequence import SPContext

    model, b = W._mmdit_setup(name)
    loss = M.mmdit_loss_local(model, b["lat"], b["noise"], b["text"], b["sig"], SPContext())
    loss.backward()
    ref_g = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1)
                       for p in model.parameters()])
    with tempfile.TemporaryDirectory() as d:
        res, _ = _run("mmdit_sp", 2, d, {"model": name, "mode": mode})
    tot = res[0]["loss"] + res[1]["loss"]
    assert tot == pytest.approx(float(loss), rel=2e-2), (tot, float(loss))
    g = res[0]["grads"] + res[1]["grads"]
    rel = ((g - ref_g).norm() / ref_g.norm()).item()
    assert rel < 2e-2, rel


def test_ring_attention_ops_two_ranks_match_sdpa():
    """The reference-compatible ring_attention_ops over two gloo ranks (K/V
    chunks gathered, dK/dV summed back to their owners): every rank's output
    and gradient chunks match SDPA over the full sequence."""
    import tempfile

    import torch.nn.functional as F

    world = 2
    g = torch.Generator().manual_seed(21)
    B, H, T, D = 1, 2, 24 * world, 32
    q, k, v, do = (torch.randn(B, H, T, D, generator=g).bfloat16() for _ in range(4))
    qf, kf, vf = (x.float().requires_grad_(True) for x in (q, k, v))
    ref = F.scaled_dot_product_attention(qf, kf, vf)
    ref.backward(do.float())
    with tempfile.TemporaryDirectory() as d:
        res, _ = _run("ring_ops_sp", world, d)
    t = T // world
    for r in range(world):
        sl = slice(r * t, (r + 1) * t)
        for key, want in (("o", ref.detach()), ("dq", qf.grad), ("dk", kf.grad), ("dv", vf.grad)):
            got = res[r][key]
            err = ((got - want[:, :, sl]).abs().max() / want[:, :, sl].abs().max()).item()
            assert err < 3e-2, (r, key, err)


@pytest.mark.skipif(not os.environ.get("HARP_REFERENCE_DIR"),
                    reason="HARP_REFERENCE_DIR (the reference project's root) not set")
def test_managers_match_the_reference_two_ranks(tmp_path):
    """Oracle: the reference's own shard_manager.py and weight_manager.py
    (pure PyTorch + torch.distributed) and harp's managers give the same
    results on two gloo ranks (forward values, input gradients, owners, row
    chunks with their gradient views, gathered parameters and ready flags)."""
    res, _ = _run("managers_oracle", 2, tmp_path, {"ref": os.environ["HARP_REFERENCE_DIR"]})
    for r in (0, 1):
        d = res[r]
        keys = sorted({k.rsplit("_", 1)[0] for k in d})
        for k in keys:
            a, b = d[k + "_ref"], d[k + "_ours"]
            if k.startswith("chunks"):
                assert len(a) == len(b), k
                for (b0, e0, v0, g0), (b1, e1, v1, g1) in zip(a, b):
                    assert (b0, e0) == (b1, e1), k
                    assert torch.equal(v0, v1), k
                    assert (g0 is None) == (g1 is None) and (g0 is None or torch.equal(g0, g1)), k
            elif isinstance(a, (list, tuple)) and a and isinstance(a[0], torch.Tensor):
                assert len(a) == len(b), k
                for u, v in zip(a, b):
                    torch.testing.assert_close(v, u, rtol=0, atol=0, msg=k)
            elif isinstance(a, torch.Tensor):
                torch.testing.assert_close(b, a, rtol=0, atol=0, msg=k)
            else:
                assert a == b, (k, a, b)


@pytest.mark.skipif(not os.environ.get("HARP_REFERENCE_DIR"),
                    reason="HARP_REFERENCE_DIR (the reference project's root) not set")
@pytest.mark.parametrize("world,hw,cap", [(1, 16, 32), (2, 16, 32), (2, 18, 20)])
def test_zimage_sp_matches_the_reference_sp_model(tmp_path, world, hw, cap):
    """Oracle: the reference's own SP Z-Image (hl_model.py, its blocks and
    attention, over the reference's standalone base model) and harp's
    Z_Transformer with harp_block_compat=True, on the same weights and inputs
    (metadata, one condition image, padded runs in the last case).  harp runs
    sequence-parallel over one or two gloo ranks (gradients summed over them);
    the reference runs on one rank (exact gradients) and, forward only, over
    the same ranks as harp.  Against the reference in fp32, harp's bf16
    predictions and gradients may deviate at most twice as much as the
    reference's own bf16 run does, plus a small floor: this model in bf16 is
    itself a few percent off fp32, more for the nearly cancelling
    caption-attention q/k gradients."""
    res, _ = _run("zimage_reference_sp", world, tmp_path,
                  {"ref": os.environ["HARP_REFERENCE_DIR"], "hw": hw, "cap": cap})

    def rel(a, b):
        return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()

    full32, full16 = res[0]["pred_ref32"], res[0]["pred_ref16"]
    for r in range(world):
        torch.testing.assert_close(res[r]["pred_ref32"], full32, rtol=0, atol=0)
        if world > 1:  # the reference's own sequence-parallel forward over these ranks
            assert rel(res[r]["pred_refw"], full16) < 1e-2, r
        lo, hi = res[r]["range"]
        ours = res[r]["pred_ours"]
        assert rel(ours, full32[:, lo:hi]) <= 2 * rel(full16[:, lo:hi], full32[:, lo:hi]) + 2e-3, r
    for n, g32 in res[0]["grads_ref32"].items():
        g16 = res[0]["grads_ref16"][n]
        ours = sum(res[r]["grads_ours"][n] for r in range(world))
        if g32.norm().item() == 0:
            assert ours.norm().item() == 0 and g16.norm().item() == 0, n
            continue
        assert rel(ours, g32) <= 2 * rel(g16, g32) + 1e-2, (n, rel(ours, g32), rel(g16, g32))


@pytest.mark.parametrize("padded,world", [(False, 2), (True, 2), (True, 4)])
def test_zimage_forward_gathers_full_predictions_two_ranks(tmp_path, padded, world):
    """Z_Transformer.forward keeps the reference's contract under sequence
    parallelism: on two or four gloo ranks every rank gets the one-process
    predictions,
    and with the loss computed in full on every rank the ranks' parameter
    gradients sum to the one-process gradients."""
    (tmp_path / "one").mkdir()
    (tmp_path / "two").mkdir()
    one, _ = _run("zimage_forward_full", 1, tmp_path / "one", {"padded": padded})
    two, _ = _run("zimage_forward_full", world, tmp_path / "two", {"padded": padded})
    for r in range(world):
        for u, v in zip(two[r]["pred"], one[0]["pred"]):
            assert ((u - v).norm() / v.norm()).item() < 2e-2
    g = sum(two[r]["grads"] for r in range(world))
    ref = one[0]["grads"]
    assert ((g - ref).norm() / ref.norm()).item() < 2e-2


@pytest.mark.parametrize("mode", ["ring", "ulysses"])
def test_zimage_gradient_checkpointing_two_ranks(tmp_path, mode):
    """With gradient checkpointing the blocks (and their sequence-parallel
    exchanges) run again in the backward on both gloo ranks: the same loss
    shares and gradients as without it."""
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    plain, _ = _run("zimage_sp", 2, tmp_path / "a", {"mode": mode, "padded": True})
    ckpt, _ = _run("zimage_sp", 2, tmp_path / "b", {"mode": mode, "padded": True, "ckpt": True})
    for r in (0, 1):
        assert ckpt[r]["loss"] == plain[r]["loss"]
        torch.testing.assert_close(ckpt[r]["grads"], plain[r]["grads"], rtol=0, atol=0)
