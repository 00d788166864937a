"""Two-GPU tests: sequence-parallel training through the NVLink kernels
(fused Ulysses and K/V gather) against one GPU, and the bounded flag wait."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

import mgpu_workers as W

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu, pytest.mark.timeout(900)]


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(name, world, tmp_path, args):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=W.entry, args=(r, world, port, name, str(tmp_path), args)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    return {r: torch.load(os.path.join(str(tmp_path), f"rank{r}.pt"), weights_only=False) for r in range(world)}


def _batch(path, n=2):
    from harp_b200.models.dit import PRESETS

    cfg = PRESETS["small"]
    g = torch.Generator().manual_seed(7)
    b = {"latent": torch.randn(n, cfg.in_channels, 32, 32, generator=g).bfloat16(),
         "noise": torch.randn(n, cfg.in_channels, 32, 32, generator=g).bfloat16(),
         "text": torch.randn(n, 64, cfg.text_dim, generator=g).bfloat16(),
         "sigmas": torch.rand(n, generator=g)}
    torch.save(b, path)
    return b


def _single(batch, steps):
    from harp_b200.models.dit import DiT, PRESETS
    from harp_b200.trainer import ParallelState, TrainConfig, Trainer

    model = DiT(PRESETS["small"])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    tr = Trainer(model, ParallelState(), TrainConfig(lr=1e-3), torch.device("cuda", 0))
    losses = [tr.step({k: v.pin_memory() for k, v in batch.items()}) for _ in range(steps)]
    return losses, torch.cat([p.detach().reshape(-1) for p in model.parameters()]).cpu()


# (sequence-parallel mode, SP exchange backend, gradient comm, overlapped bucketed gradient sync,
#  parameters per bucket, sharded block weights): the 1M buckets put about one block in each
#  bucket of the small preset
@pytest.mark.parametrize("mode,backend,comm,overlap,bucket,shard", [
    ("ulysses", "nvl", "nvl", True, 1_000_000, False), ("ring", "nvl", "nvl", True, 64_000_000, False),
    ("ulysses", "nvl", "nvl", False, 1_000_000, False), ("ulysses", "torch", "torch", False, 64_000_000, False),
    ("ulysses", "nvl", "nvl", True, 64_000_000, True), ("ring", "nvl", "nvl", True, 64_000_000, True)])
def test_sp2_training_matches_one_gpu(tmp_path, mode, backend, comm, overlap, bucket, shard):
    _need(2)
    bpath = str(tmp_path / "batch.pt")
    batch = _batch(bpath)
    ref_losses, ref_flat = _single(batch, 3)
    res = _run("train", 2, tmp_path, {"batch": bpath, "steps": 3, "mode": mode, "backend": backend, "comm": comm,
                                      "overlap": overlap, "bucket_params": bucket, "shard": shard})
    for r in (0, 1):
        assert res[r]["mode"] == mode and res[r]["backend"] == backend
        assert res[r]["overlap"] == ((overlap or shard) and comm == "nvl") and res[r]["buckets"] > 1, res[r]
        assert res[r]["losses"] == pytest.approx(ref_losses, rel=1e-2), (res[r]["losses"], ref_losses)
        torch.testing.assert_close(res[r]["flat"].float(), ref_flat.float(), rtol=2 ** -6, atol=2 * 3 * 1e-3)
    assert torch.equal(res[0]["flat"], res[1]["flat"])


@pytest.mark.parametrize("mode,shard", [("ulysses", False), ("ring", True)])
def test_sp2_cuda_graph_step_matches_eager(tmp_path, monkeypatch, mode, shard):
    """The whole 2-GPU step captured once and replayed (flag values advanced on
    the device per replay) follows the eager steps.  The attention backward
    accumulates dQ with reduce-adds in no fixed order, so two runs agree to
    rounding, not bit for bit; the ranks' replicated parameters stay identical."""
    _need(2)
    bpath = str(tmp_path / "batch.pt")
    _batch(bpath)
    res = {}
    monkeypatch.setenv("HARP_GRAPH_MULTI", "1")
    for graph in (False, True):
        d = tmp_path / f"g{int(graph)}"
        d.mkdir()
        res[graph] = _run("train", 2, d, {"batch": bpath, "steps": 8, "mode": mode, "backend": "nvl", "comm": "nvl",
                                          "overlap": True, "bucket_params": 1_000_000, "shard": shard,
                                          "graph": graph})
    for r in (0, 1):
        assert res[True][r]["graph_replays"] == 6, res[True][r]["graph_replays"]
        assert res[True][r]["losses"][:2] == res[False][r]["losses"][:2]  # the same eager steps
        assert res[True][r]["losses"] == pytest.approx(res[False][r]["losses"], rel=1e-3), \
            (res[True][r]["losses"], res[False][r]["losses"])
        torch.testing.assert_close(res[True][r]["flat"].float(), res[False][r]["flat"].float(), rtol=2 ** -7,
                                   atol=2e-3)
    assert torch.equal(res[True][0]["flat"], res[True][1]["flat"])


def test_nvlink_exchange_kernels_on_one_rank(tmp_path):
    """The fused Ulysses and ring exchange kernels on a one-GPU group (the peer
    tables hold this GPU's own buffers), so they also run where only one GPU
    is present: attention forward and backward through them match fp32 SDPA."""
    _need(1)
    res = _run("nvl_world1", 1, tmp_path, {})[0]
    for key, err in res.items():
        assert err < 2e-2, (key, err, res)


def test_never_signalled_flag_times_out_cleanly(tmp_path):
    _need(2)
    res = _run("flag_timeout", 2, tmp_path, {})
    for r in (0, 1):
        assert res[r]["err"][0] == 2 and res[r]["err"][1] >= 100, res[r]  # peer timeout at a wait site
        assert res[r]["x"] == 8.0


def test_harp_nvl_c10d_backend_collectives(tmp_path):
    _need(2)
    res = _run("c10d_backend", 2, tmp_path, {})
    for r in (0, 1):
        d = res[r]
        for k, v in d.items():
            if k.startswith("ar_"):
                assert v < 1e-2, (r, k, v)
        assert d["max"] == 1.0
        assert d["ag"] and d["rs"] and d["bcast"] and d["a2a"] and d["async"], d
        assert d["ag_list"] == [[0.5] * 3, [1.5] * 3]
