"""Host-side utilities: scheduler and loss weighting, learning-rate schedules,
the .npz data format, logging / timing, fault injection, heartbeat, the wait
and copy engines (reference test strategy: each helper checked in isolation
against closed-form values)."""
import json
import math
import os
import time

import numpy as np
import pytest
import torch

from harp_b200.managers import mem_manager as MM
from harp_b200.managers import ring_attn_manager as RA
from harp_b200.utils import data as DA
from harp_b200.utils import diffusion as DF
from harp_b200.utils import fault as FT
from harp_b200.utils import observability as OB


def test_flow_match_scheduler_shift_and_lookup(tmp_path):
    s = DF.FlowMatchEulerDiscreteScheduler(num_train_timesteps=1000, shift=3.0)
    t = torch.linspace(1000, 1, 1000) / 1000
    ref = 3.0 * t / (1 + 2.0 * t)
    torch.testing.assert_close(s.sigmas, ref)
    torch.testing.assert_close(s.timesteps, ref * 1000)
    idx = torch.tensor([0, 10, 999])
    torch.testing.assert_close(s.sigmas_for(s.timesteps[idx]), s.sigmas[idx])
    s.save_config(str(tmp_path / "scheduler"))
    s2 = DF.FlowMatchEulerDiscreteScheduler.from_pretrained(str(tmp_path), subfolder="scheduler")
    assert s2.config.shift == 3.0
    torch.testing.assert_close(s2.sigmas, s.sigmas)
    # missing config directory: defaults (the reference loads diffusers' defaults)
    assert DF.FlowMatchEulerDiscreteScheduler.from_pretrained(str(tmp_path / "nope")).config.shift == 1.0


def test_timestep_density_and_weighting():
    g = torch.Generator().manual_seed(0)
    for scheme in ("logit_normal", "mode", "none", "sigma_sqrt", "cosmap"):
        u = DF.compute_density_for_timestep_sampling(scheme, 4096, 0.0, 1.0, 1.29, generator=g)
        assert u.shape == (4096,) and (u >= 0).all() and (u <= 1).all(), scheme
    u = DF.compute_density_for_timestep_sampling("logit_normal", 20000, 0.0, 1.0, generator=g)
    assert abs(u.mean().item() - 0.5) < 0.01  # sigmoid of a symmetric normal
    sig = torch.tensor([0.25, 0.5, 1.0])
    torch.testing.assert_close(DF.compute_loss_weighting_for_sd3("sigma_sqrt", sig), sig ** -2.0)
    torch.testing.assert_close(DF.compute_loss_weighting_for_sd3("cosmap", sig),
                               2 / (math.pi * (1 - 2 * sig + 2 * sig ** 2)))
    torch.testing.assert_close(DF.compute_loss_weighting_for_sd3("logit_normal", sig), torch.ones(3))


@pytest.mark.parametrize("name", ["constant", "constant_with_warmup", "linear", "cosine", "cosine_with_restarts",
                                  "polynomial"])
def test_lr_schedules_closed_form(name):
    W, T, base = 10, 100, 1e-3
    sch = DF.LRSchedule(name, base, num_warmup_steps=W, num_training_steps=T)
    lrs = []
    for _ in range(T):
        lrs.append(sch.lr())
        sch.step()
    if name != "constant":
        assert lrs[0] == 0.0 and abs(lrs[5] - base * 0.5) < 1e-12
    if name == "linear":
        assert abs(lrs[55] - base * (T - 55) / (T - W)) < 1e-12
    if name == "cosine":
        assert abs(lrs[55] - base * 0.5 * (1 + math.cos(math.pi * 45 / 90))) < 1e-12
    # state round trip
    sd = sch.state_dict()
    sch2 = DF.LRSchedule(name, base, num_warmup_steps=W, num_training_steps=T)
    sch2.load_state_dict(sd)
    assert sch2.lr() == sch.lr()


def test_piecewise_constant_rules():
    sch = DF.LRSchedule("piecewise_constant", 1.0, step_rules="1:10,0.1:20,0.01")
    got = []
    for _ in range(30):
        got.append(sch.lr())
        sch.step()
    assert got[0] == 1.0 and got[10] == pytest.approx(0.1) and got[25] == pytest.approx(0.01)


def test_npz_dataset_roundtrip_and_collate(tmp_path):
    idx = DA.write_npz_samples(str(tmp_path), 3, latent_channels=4, latent_size=8, text_len=5, text_dim=6,
                               num_metadata=4, cond_channels=3)
    ds = DA.NpzDataset(idx)
    assert len(ds) == 3 and ds.num_metadata == 4
    it = ds[1]
    assert it["latent_image"].shape == (4, 8, 8) and it["prompt_embeds"].shape == (5, 6)
    # a path whose directories do not exist is found by name next to the index
    with open(idx) as fh:
        names = json.load(fh)
    with open(idx, "w") as fh:
        json.dump(["HARP/data/" + n for n in names], fh)
    ds2 = DA.NpzDataset(str(tmp_path))
    np.testing.assert_array_equal(ds2[1]["latent_image"], it["latent_image"])
    b = DA.collate([ds[0], ds[1]])
    assert b["latent_image"].shape == (2, 4, 8, 8)
    assert isinstance(b["prompt_embeds"], list) and len(b["prompt_embeds"]) == 2
    assert b["norm_metadata"].shape == (2, 4)
    assert isinstance(b["cond"], list) and b["cond"][0].shape == (2, 3, 8, 8)
    assert DA.custom_collate_fn is DA.collate and DA.TiffDataset is DA.NpzDataset


def test_synthetic_data_is_deterministic():
    a = DA.SyntheticDiTData(4, 4, 8, 5, 6, num_metadata=2, cond_channels=3, seed=7)
    b = DA.SyntheticDiTData(4, 4, 8, 5, 6, num_metadata=2, cond_channels=3, seed=7)
    for k in a[2]:
        np.testing.assert_array_equal(a[2][k], b[2][k])
    assert not np.array_equal(a[1]["latent_image"], a[2]["latent_image"])


def test_logger_phase_timer_and_jsonl(tmp_path):
    log = OB.setup_logger(str(tmp_path / "train.log"), True)
    log.info("hello")
    for h in log.handlers:
        h.flush()
    assert "hello" in (tmp_path / "train.log").read_text()
    t = OB.PhaseTimer()
    with t.phase("a"):
        time.sleep(0.01)
    with t.phase("a"):
        pass
    rep = t.report()
    assert rep["a"] >= 9.0
    w = OB.JsonlWriter(str(tmp_path / "m" / "metrics.jsonl"))
    w.write({"x": 1})
    w.write({"x": 2})
    lines = (tmp_path / "m" / "metrics.jsonl").read_text().splitlines()
    assert [json.loads(l)["x"] for l in lines] == [1, 2]
    with OB.nvtx("noop"):
        pass


def test_fault_injector_kinds(monkeypatch):
    f = FT.FaultInjector("raise@step:3,delay_ms@signal:20,drop@grad_sync", rank=0)
    assert f.fire("step", 2)
    with pytest.raises(FT.HarpInjectedFault):
        f.fire("step", 3)
    t0 = time.time()
    assert f.fire("signal")
    assert time.time() - t0 >= 0.015
    assert f.fire("grad_sync") is False  # dropped once
    assert f.fire("grad_sync") is True
    monkeypatch.setenv("HARP_FAULT_RANK", "1")
    g = FT.FaultInjector("raise@step", rank=0)
    assert g.fire("step", 0)  # only rank 1 is faulty


def test_heartbeat_detects_stopped_rank():
    store = torch.distributed.HashStore()
    hb0 = FT.Heartbeat(store, 0, 2, period_s=0.05)
    hb1 = FT.Heartbeat(store, 1, 2, period_s=0.05)
    time.sleep(0.2)
    assert hb0.stale(0.15) == []
    hb1.stop()
    hb0.stale(0.15)
    time.sleep(0.4)
    assert hb0.stale(0.15) == [1]
    hb0.stop()


def test_wait_engine_completion_and_failure():
    eng = RA.CPUWaitEngine()
    try:
        class Req:
            def __init__(self, ok):
                self.ok = ok

            def wait(self):
                time.sleep(0.01)
                if not self.ok:
                    raise RuntimeError("peer gone")

        w = eng.submit(Req(True))
        assert w.wait(timeout=5) and w.is_completed()
        bad = eng.submit(Req(False))
        with pytest.raises(RuntimeError):
            bad.wait(timeout=5)
    finally:
        eng.shutdown()


def test_memory_tiers_and_copy_engine_on_cpu():
    with MM.use_hbm_allocator(False):
        assert not MM.on_hbm()
        with MM.use_hbm_allocator(True):
            assert MM.on_hbm()
        assert not MM.on_hbm()
    x = MM.empty(4, 4, dtype=torch.float32, device="cpu")
    assert x.shape == (4, 4)
    eng = MM.CopyEngine.get_instance()
    src = torch.randn(16)
    w = eng.submit(src, to_host=True)
    torch.testing.assert_close(w.wait(), src)
    off = MM.HBMToDDROffloader()
    with torch.autograd.graph.saved_tensors_hooks(off.pack_hook, off.unpack_hook):
        a = torch.randn(8, requires_grad=True)
        (a * a).sum().backward()
    torch.testing.assert_close(a.grad, 2 * a.detach())
    eng.shutdown()


def test_metadata_roundtrip_and_caption():
    from harp_b200.utils.misc import MetaData

    md = MetaData()
    raw = (120.5, -33.25, 0.5, 2020.0)
    n = md.normalize(raw)
    torch.testing.assert_close(n, torch.tensor([120.5 / 360 * 1000, -33.25 / 180 * 1000, 50.0, 2020 / 2100 * 1000]))
    torch.testing.assert_close(md.unnormalize(n), torch.tensor(raw))
    emb, cap = md.embedding(raw)
    assert "resolution of 0.5" in cap and "2020.0" in cap


def test_apply_rotary_emb_real_and_complex_agree():
    from harp_b200.utils.misc import apply_rotary_emb

    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 3, 5, 8, generator=g)
    ang = torch.randn(2, 5, 4, generator=g)
    cis = torch.polar(torch.ones_like(ang), ang)
    cos = ang.cos().repeat_interleave(2, -1)
    sin = ang.sin().repeat_interleave(2, -1)
    a = apply_rotary_emb(x, (cos, sin), use_real=True)
    b = apply_rotary_emb(x, cis, use_real=False)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    # rotation keeps the norm of every pair
    torch.testing.assert_close(a.norm(dim=-1), x.norm(dim=-1), rtol=1e-5, atol=1e-5)


def test_fast_init_mode_is_deterministic():
    from harp_b200.utils.misc import FastInitMode

    def build():
        with FastInitMode(seed=7):
            return torch.nn.Linear(16, 8)

    a, b = build(), build()
    assert torch.equal(a.weight, b.weight) and torch.equal(a.bias, b.bias)
    bound = 1 / math.sqrt(16)
    assert a.weight.abs().max() <= bound


def test_save_trainable_param_hook(tmp_path):
    from safetensors.torch import load_file

    from harp_b200.utils.misc import preserve_requires_grad, save_trainable_param_hook

    m = torch.nn.Sequential(torch.nn.Linear(4, 4), torch.nn.Linear(4, 2))
    m[0].weight.requires_grad_(False)
    save_trainable_param_hook([m], [1], str(tmp_path))
    sd = load_file(str(tmp_path / "model.safetensors"))
    assert set(sd) == {"0.bias", "1.weight", "1.bias"}
    with preserve_requires_grad(m):
        m.requires_grad_(False)
    assert m[1].weight.requires_grad and not m[0].weight.requires_grad


def test_launch_rankfile_cpu_sets_and_command(tmp_path):
    from harp_b200 import launch as L

    lines = L.generate_rankfile(["node10", "node2", "node2"], ranks_per_node=2, cores_per_node=8)
    assert lines == ["rank 0=node2 gpu=0 cpus=0-3", "rank 1=node2 gpu=1 cpus=4-7",
                     "rank 2=node10 gpu=0 cpus=0-3", "rank 3=node10 gpu=1 cpus=4-7"]
    # two GPUs per NUMA node: each rank gets half of its node's cores
    aff = {0: [0, 1, 2, 3], 1: [0, 1, 2, 3], 2: [4, 5, 6, 7], 3: [4, 5, 6, 7]}
    assert L.cpu_sets(4, affinity=aff) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    cmd = L.torchrun_cmd(["train.py", "--x"], 8)
    assert "--master-addr=127.0.0.1" in cmd and cmd[-2:] == ["train.py", "--x"]


def test_train_cli_checkpoint_and_resume_bit_exact(tmp_path):
    """train.py end to end on CPU (tiny DiT, synthetic data): a 3-step run saves
    checkpoint-2 and logs metrics; a second run with --resume_from_checkpoint
    latest continues at step 3 with the same loss, bit for bit."""
    import json
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    work = str(tmp_path / "w")
    base = [sys.executable, os.path.join(root, "train.py"), "--model", "tiny", "--synthetic", "--latent_size", "16",
            "--text_len", "16", "--max_train_steps", "3", "--train_batch_size", "2", "--sp_size", "1",
            "--work_dir", work, "--checkpointing_steps", "2", "--lr_warmup_steps", "1"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")

    def losses(out_dir):
        rows = [json.loads(l) for l in open(os.path.join(out_dir, "metrics.jsonl")) if l.strip()]
        return {r["global_step"]: r["step_loss"] for r in rows if "step_loss" in r}

    r1 = subprocess.run(base, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert r1.returncode == 0, r1.stderr[-3000:]
    runs = sorted(os.listdir(work))
    assert len(runs) == 1 and os.path.isdir(os.path.join(work, runs[0], "checkpoint-2"))
    first = losses(os.path.join(work, runs[0]))
    assert sorted(first) == [1, 2, 3]
    r2 = subprocess.run(base + ["--resume_from_checkpoint", "latest"], capture_output=True, text=True, timeout=600,
                        env=env, cwd=str(tmp_path))
    assert r2.returncode == 0, r2.stderr[-3000:]
    metrics = [os.path.join(d, "metrics.jsonl") for d, _, files in os.walk(work) if "metrics.jsonl" in files]
    second_runs = [m for m in metrics if os.path.dirname(m) != os.path.join(work, runs[0])]
    assert len(second_runs) == 1, metrics
    second = losses(os.path.dirname(second_runs[0]))
    assert sorted(second) == [3] and second[3] == first[3], (first, second)


def test_train_cli_two_ranks_checkpoint_resume(tmp_path):
    """train.py under torchrun with two gloo ranks (2-way sequence parallel):
    every rank's optimizer shard is saved, and the resumed run's next step has
    the loss of the uninterrupted run, bit for bit."""
    import socket
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    work = str(tmp_path / "w")

    def cmd(extra):
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(root, "train.py"),
                "--model", "tiny", "--synthetic", "--latent_size", "16", "--text_len", "16", "--max_train_steps", "3",
                "--train_batch_size", "2", "--sp_size", "2", "--work_dir", work, "--checkpointing_steps", "2",
                "--lr_warmup_steps", "1"] + extra

    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r1 = subprocess.run(cmd([]), capture_output=True, text=True, timeout=900, env=env, cwd=str(tmp_path))
    assert r1.returncode == 0, r1.stderr[-3000:]
    (run,) = os.listdir(work)
    ck = os.path.join(work, run, "checkpoint-2")
    assert {"optimizer.rank0.bin", "optimizer.rank1.bin", "pytorch_model.bin"} <= set(os.listdir(ck))
    first = {r["global_step"]: r["step_loss"] for r in map(json.loads, open(os.path.join(work, run, "metrics.jsonl")))
             if "step_loss" in r}
    r2 = subprocess.run(cmd(["--resume_from_checkpoint", "latest"]), capture_output=True, text=True, timeout=900,
                        env=env, cwd=str(tmp_path))
    assert r2.returncode == 0, r2.stderr[-3000:]
    second = {r["global_step"]: r["step_loss"] for r in map(json.loads, open(os.path.join(work, "metrics.jsonl")))
              if "step_loss" in r}
    assert sorted(second) == [3] and second[3] == first[3], (first, second)


def test_async_runtime_api_on_streams():
    """The reference's async-runtime API (async_rt/): the mode switches and
    syncs are identities on values and gradients and set the mode flag as the
    reference's do; MyMul / MyAdd broadcast and sum gradients back to each
    input's shape; the kernel helpers write the linear and SiLU results into
    the caller's tensors (CPU restatements here, to bf16 rounding)."""
    from harp_b200.compat import install_reference_import_paths

    install_reference_import_paths()
    import async_rt
    from async_rt import async_ops as O
    from async_rt import runtime as R

    assert async_rt.is_asyncrt_enabled() is False
    x = torch.randn(2, 3, requires_grad=True)
    y = R.AsyncModeStart.apply(x)
    assert R.AsyncRunMode.mode_enable is True
    y = R.AsyncSync.apply(y, True, True)
    y = R.AsyncModeEnd.apply(y)
    assert R.AsyncRunMode.mode_enable is False
    (y * 3).sum().backward()
    torch.testing.assert_close(x.grad, torch.full_like(x, 3.0))
    R.RUNTIME.sync()
    with R.AsyncRunMode():
        torch.testing.assert_close(torch.ones(2) + 1, torch.full((2,), 2.0))

    a = torch.randn(4, 1, 5, requires_grad=True)
    b = torch.randn(3, 5, requires_grad=True)
    O.MyMul.apply(a, b).pow(2).sum().backward()
    ga, gb = a.grad.clone(), b.grad.clone()
    a.grad = b.grad = None
    (a * b).pow(2).sum().backward()
    torch.testing.assert_close(ga, a.grad)
    torch.testing.assert_close(gb, b.grad)
    a.grad = b.grad = None
    O.MyAdd.apply(a, b).pow(2).sum().backward()
    ga, gb = a.grad.clone(), b.grad.clone()
    a.grad = b.grad = None
    (a + b).pow(2).sum().backward()
    torch.testing.assert_close(ga, a.grad)
    torch.testing.assert_close(gb, b.grad)
    b.grad = None
    O.MyAdd.apply(2.5, b).sum().backward()
    torch.testing.assert_close(b.grad, torch.ones_like(b))

    torch.manual_seed(0)
    xin = torch.randn(6, 16).bfloat16()
    w = torch.randn(8, 16).bfloat16()
    bias = torch.randn(8).bfloat16()
    out = torch.empty(6, 8, dtype=torch.bfloat16)
    O.mm_kernel(out, xin, w, bias)
    ref = xin.float() @ w.float().t() + bias.float()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    dy = torch.randn(6, 8).bfloat16()
    gi, gw, gbias = torch.empty_like(xin), torch.empty_like(w), torch.empty_like(bias)
    O.mm_backward_kernel(gi, dy, xin, w, gw, gbias)
    torch.testing.assert_close(gi.float(), dy.float() @ w.float(), rtol=2e-2, atol=5e-2)
    torch.testing.assert_close(gw.float(), dy.float().t() @ xin.float(), rtol=2e-2, atol=5e-2)
    torch.testing.assert_close(gbias.float(), dy.float().sum(0), rtol=2e-2, atol=5e-2)
    s = torch.empty_like(xin)
    O.silu_kernel(s, xin)
    torch.testing.assert_close(s.float(), torch.nn.functional.silu(xin.float()), rtol=1e-2, atol=1e-2)
    O.silu_backward_kernel(s, dy[:, :1].expand(6, 16).contiguous(), xin)
    xf = xin.float().requires_grad_(True)
    torch.nn.functional.silu(xf).backward(dy[:, :1].expand(6, 16).float())
    torch.testing.assert_close(s.float(), xf.grad, rtol=1e-2, atol=1e-2)
    o2 = torch.empty(6, 16)
    O.mul_fast(o2, xin.float(), xin.float())
    torch.testing.assert_close(o2, xin.float() ** 2)
    O.add_kernel(o2, xin.float(), xin.float())
    torch.testing.assert_close(o2, 2 * xin.float())


def test_reference_import_paths():
    """harp_b200.compat registers the reference's top-level import paths
    (managers.*, async_rt.*, unigemm_linear, kp_normalization,
    kp_multi_tensor_adamw, kp_rope, kp_rope_embedder) as harp's modules, and
    every name the reference imports from them resolves."""
    import importlib

    from harp_b200.compat import REFERENCE_MODULES, install_reference_import_paths
    from harp_b200.models import zimage as Z
    from harp_b200.ops import modules as M

    install_reference_import_paths()
    for name, target in REFERENCE_MODULES.items():
        assert importlib.import_module(name) is importlib.import_module(target), name
    want = {
        "unigemm_linear": {"kpLinear": M.kpLinear, "replace_linear_with_kplinear": M.replace_linear_with_kplinear,
                           "CustomLinearFunction": M.LinearFunction},
        "kp_normalization": {"kpRMSNorm": M.kpRMSNorm, "CustomNormFunction": M.RMSNormFunction,
                             "replace_rmsNorm_with_kpRMSNorm": M.replace_rmsNorm_with_kpRMSNorm},
        "kp_multi_tensor_adamw": {"kp_multi_tensor_adamw": M.kp_multi_tensor_adamw},
        "kp_rope": {"kp_apply_rotary_emb": M.kp_apply_rotary_emb},
        "kp_rope_embedder": {"RopeEmbedderSVE": Z.RopeTableEmbedder, "RopeEmbedderReference": Z.RopeEmbedder,
                             "replace_ropeembedder_with_sverope": Z.replace_ropeembedder_with_sverope},
        "async_rt.async_ops": {"MySiLU": M.MySiLU, "MyTanh": M.MyTanh, "ApplyRotaryComplexFn": M.ApplyRotaryComplexFn},
    }
    for mod_name, names in want.items():
        mod = importlib.import_module(mod_name)
        for n, obj in names.items():
            assert getattr(mod, n) is obj, (mod_name, n)
    # every `from X import a, b` of the reference's train.py and Z-Image SP model
    from async_rt import is_asyncrt_enabled  # noqa: F401
    from async_rt.async_ops import MySiLU  # noqa: F401
    from async_rt.runtime import RUNTIME, AsyncModeEnd, AsyncModeStart, AsyncRunMode, AsyncSync  # noqa: F401
    from managers.grad_manager import AsyncGradSyncManager  # noqa: F401
    from managers.mem_manager import use_hbm_allocator  # noqa: F401
    from managers.ring_attn_manager import CPUWaitEngine  # noqa: F401
    from managers.shard_manager import SequenceAllGather, SequenceScatter, SPBroadcast  # noqa: F401
    from managers.weight_manager import (AsyncParamAllGatherManager, build_balanced_param_groups,  # noqa: F401
                                         build_chunk_param, set_opt_hook, setup_shared_model)


def test_train_cli_under_mpirun_style_environment(tmp_path):
    """train.py started the way mpirun starts it (OMPI_COMM_WORLD_RANK / _SIZE /
    _LOCAL_RANK in the environment, no torchrun variables): two processes
    find each other, train two sequence-parallel steps over gloo and write one
    metrics file."""
    import json
    import socket
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    work = tmp_path / "w"
    cmd = [sys.executable, os.path.join(root, "train.py"), "--model", "tiny", "--synthetic", "--latent_size", "16",
           "--text_len", "16", "--max_train_steps", "2", "--train_batch_size", "2", "--sp_size", "2",
           "--work_dir", str(work), "--checkpointing_steps", "100", "--lr_warmup_steps", "1"]
    base = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR",
                                                             "MASTER_PORT")}
    procs = []
    for r in range(2):
        env = dict(base, CUDA_VISIBLE_DEVICES="", OMPI_COMM_WORLD_RANK=str(r), OMPI_COMM_WORLD_SIZE="2",
                   OMPI_COMM_WORLD_LOCAL_RANK=str(r), MASTER_PORT=str(port))
        procs.append(subprocess.Popen(cmd, env=env, cwd=str(tmp_path), stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=600) for p in procs]
    for p, (_, err) in zip(procs, outs):
        assert p.returncode == 0, err[-3000:]
    (run,) = os.listdir(work)
    rows = [json.loads(line) for line in open(work / run / "metrics.jsonl") if line.strip()]
    assert [row["global_step"] for row in rows if "step_loss" in row] == [1, 2]


def test_reference_import_paths_leave_a_foreign_package_alone(monkeypatch):
    """A package already imported under a reference name (for example the
    reference's own `managers`) keeps that name and its submodules unless
    replace=True."""
    import sys
    import types

    from harp_b200.compat import REFERENCE_MODULES, install_reference_import_paths
    from harp_b200.managers import shard_manager

    for name in REFERENCE_MODULES:
        monkeypatch.delitem(sys.modules, name, raising=False)
    foreign = types.ModuleType("managers")
    monkeypatch.setitem(sys.modules, "managers", foreign)
    done = install_reference_import_paths()
    assert sys.modules["managers"] is foreign and "managers.shard_manager" not in sys.modules
    assert not any(n.startswith("managers") for n in done) and "async_rt" in done
    done = install_reference_import_paths(replace=True)
    assert sys.modules["managers.shard_manager"] is shard_manager and "managers" in done
