"""Oracle tests against the reference's own pure-PyTorch modules.

The reference project's root is read from HARP_REFERENCE_DIR; every test here
is skipped when it is unset.  Files are loaded one at a time with importlib
and none of the reference's compiled extensions are needed: most import
nothing but torch and the standard library; src/utils/inference.py gets
stand-ins for the diffusers names it imports.  Each test runs the reference's
code and harp's on the same inputs (train.py and data/ are read, not run).
"""
import importlib.util
import json
import math
import os

import pytest
import torch

REF = os.environ.get("HARP_REFERENCE_DIR")
pytestmark = pytest.mark.skipif(not REF, reason="HARP_REFERENCE_DIR (the reference project's root) not set")


def _load(rel):
    spec = importlib.util.spec_from_file_location("_reference_" + rel.replace("/", "_")[:-3],
                                                  os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _lrs(get, name, **kw):
    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1e-3)
    sched = get(name, opt, **kw)
    out = []
    for _ in range(60):
        out.append(opt.param_groups[0]["lr"])
        opt.step()
        sched.step()
    return out


@pytest.mark.parametrize("name,kw", [
    ("constant", {}),
    ("constant_with_warmup", dict(num_warmup_steps=7)),
    ("piecewise_constant", dict(step_rules="1:10,0.1:20,0.01")),
    ("linear", dict(num_warmup_steps=5, num_training_steps=50)),
    ("cosine", dict(num_warmup_steps=5, num_training_steps=50)),
    ("cosine_with_restarts", dict(num_warmup_steps=5, num_training_steps=50, num_cycles=3)),
    ("polynomial", dict(num_warmup_steps=5, num_training_steps=50, power=2.0)),
])
def test_lr_schedules(name, kw):
    """src/utils/standalone_diffusion.py:92-250 (get_scheduler and the seven
    schedules) against harp_b200.utils.diffusion.get_scheduler: the learning
    rate of 60 steps, past the end of training."""
    from harp_b200.utils import diffusion as D

    R = _load("src/utils/standalone_diffusion.py")
    assert _lrs(D.get_scheduler, name, **kw) == pytest.approx(_lrs(R.get_scheduler, name, **kw), rel=1e-12, abs=0)


def test_lr_schedule_argument_errors():
    """The reference refuses a warm-up schedule without num_warmup_steps and a
    decaying one without num_training_steps; so does harp."""
    from harp_b200.utils import diffusion as D

    R = _load("src/utils/standalone_diffusion.py")
    for get in (R.get_scheduler, D.get_scheduler):
        opt = torch.optim.SGD([torch.nn.Parameter(torch.zeros(1))], lr=1e-3)
        with pytest.raises(ValueError):
            get("constant_with_warmup", opt)
        with pytest.raises(ValueError):
            get("cosine", opt, num_warmup_steps=3)


@pytest.mark.parametrize("scheme", ["logit_normal", "mode", "uniform"])
def test_timestep_density_and_loss_weighting(scheme):
    """standalone_diffusion.py:253-281: the same generator draws the same u;
    the SD3 loss weights agree."""
    from harp_b200.utils import diffusion as D

    R = _load("src/utils/standalone_diffusion.py")
    kw = dict(logit_mean=0.3, logit_std=1.2, mode_scale=1.29)
    a = R.compute_density_for_timestep_sampling(scheme, 64, generator=torch.Generator().manual_seed(5), **kw)
    b = D.compute_density_for_timestep_sampling(scheme, 64, generator=torch.Generator().manual_seed(5), **kw)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    sig = torch.linspace(0.05, 1.0, 40)
    for w in ("sigma_sqrt", "cosmap", "none"):
        torch.testing.assert_close(R.compute_loss_weighting_for_sd3(w, sig), D.compute_loss_weighting_for_sd3(w, sig))


@pytest.mark.parametrize("shift", [1.0, 3.0])
def test_flow_match_scheduler_tables_and_config(tmp_path, shift):
    """standalone_diffusion.py:23-89: the training timesteps and sigmas, their
    ends, and from_pretrained on a scheduler_config.json."""
    from harp_b200.utils import diffusion as D

    R = _load("src/utils/standalone_diffusion.py")
    a, b = R.FlowMatchEulerDiscreteScheduler(shift=shift), D.FlowMatchEulerDiscreteScheduler(shift=shift)
    torch.testing.assert_close(a.timesteps, b.timesteps)
    torch.testing.assert_close(a.sigmas, b.sigmas[:len(a.sigmas)])
    assert (a.sigma_min, a.sigma_max) == pytest.approx((b.sigma_min, b.sigma_max))
    cfg = {"num_train_timesteps": 500, "shift": shift, "base_shift": 0.4, "use_dynamic_shifting": False}
    (tmp_path / "scheduler").mkdir()
    (tmp_path / "scheduler" / "scheduler_config.json").write_text(json.dumps(cfg))
    a = R.FlowMatchEulerDiscreteScheduler.from_pretrained(str(tmp_path), subfolder="scheduler")
    b = D.FlowMatchEulerDiscreteScheduler.from_pretrained(str(tmp_path), subfolder="scheduler")
    torch.testing.assert_close(a.timesteps, b.timesteps)
    for k in cfg:
        assert a.config[k] == b.config[k]


def test_timestep_embeddings():
    """src/models/embedding.py:7-158: sinusoidal embeddings under every flag,
    and TimestepEmbedding / TimestepEmbedder on shared weights (harp's MLPs run
    on its GEMM, whose output is bf16)."""
    from harp_b200.models import embedding as E

    R = _load("src/models/embedding.py")
    t = torch.rand(9) * 1000
    for dim in (256, 255, 64):
        for flip in (False, True):
            for shift in (0.0, 1.0):
                for scale in (1.0, 3.0):
                    torch.testing.assert_close(
                        E.get_timestep_embedding(t, dim, flip, shift, scale, 5000),
                        R.get_timestep_embedding(t, dim, flip, shift, scale, 5000), rtol=0, atol=2e-6)
        torch.testing.assert_close(E.Timesteps(dim, True, 0.0)(t), R.Timesteps(dim, True, 0.0)(t), rtol=0, atol=2e-6)
    torch.manual_seed(0)
    for act, post in (("silu", None), ("gelu", "mish")):
        ref = R.TimestepEmbedding(64, 96, act, 80, post, cond_proj_dim=32)
        ours = E.TimestepEmbedding(64, 96, act, 80, post, cond_proj_dim=32)
        ours.load_state_dict(ref.state_dict())
        x, c = torch.randn(5, 64), torch.randn(5, 32)
        a, b = ref(x, c), ours(x, c).float()
        assert ((a - b).abs().max() / a.abs().max()).item() < 2e-2
    ref, ours = R.TimestepEmbedder(128, 256), E.TimestepEmbedder(128, 256)
    ours.load_state_dict(ref.state_dict())
    a, b = ref(t), ours(t).float()
    assert ((a - b).abs().max() / a.abs().max()).item() < 2e-2


@pytest.mark.parametrize("form", ["2d", "3d", "4d1", "4dh", "halves", "complex"])
def test_apply_rotary_emb(form):
    """src/utils/rope.py:6-66 against harp_b200.utils.misc.apply_rotary_emb for
    every frequency layout."""
    from harp_b200.utils.misc import apply_rotary_emb

    R = _load("src/utils/rope.py")
    B, H, S, D = 2, 3, 10, 16
    x = torch.randn(B, H, S, D).bfloat16()
    ang = torch.rand(B, S, D // 2) * 6
    if form == "complex":
        f = torch.polar(torch.ones_like(ang), ang)
        kw = dict(use_real=False)
    else:
        half = form == "halves"
        cos = torch.cat([ang.cos(), ang.cos()], -1) if half else ang.cos().repeat_interleave(2, -1)
        sin = torch.cat([ang.sin(), ang.sin()], -1) if half else ang.sin().repeat_interleave(2, -1)
        if form == "2d":
            cos, sin = cos[0], sin[0]
        elif form == "4d1":
            cos, sin = cos[:, None], sin[:, None]
        elif form == "4dh":
            cos, sin = cos[:, None].expand(B, H, S, D), sin[:, None].expand(B, H, S, D)
        f = (cos, sin)
        kw = dict(use_real=True, use_real_unbind_dim=-2 if half else -1)
    want = R.apply_rotary_emb(x, f, **kw)
    got = apply_rotary_emb(x, f, **kw)
    torch.testing.assert_close(got.float(), want.float(), rtol=0, atol=0)


def test_rope_embedder_tables():
    """kp_rope_embedder.py:6-44 (the reference's table lookup) against harp's
    RopeEmbedder, which computes the angles directly: same complex
    frequencies at every id."""
    from harp_b200.models.zimage import RopeEmbedder

    R = _load("kp_rope_embedder.py")
    dims, lens = (32, 48, 48), (1024, 512, 512)
    ref = R.RopeEmbedderReference(256.0, dims, lens)
    ids = torch.stack([torch.randint(0, n, (300,)) for n in lens], -1).int()
    from harp_b200.models.zimage import RopeTableEmbedder

    for cls in (RopeEmbedder, RopeTableEmbedder):
        torch.testing.assert_close(cls(256.0, dims, lens).complex(ids), ref(ids), rtol=0, atol=2e-6)


def test_kp_rope_complex_form():
    """kp_apply_rotary_emb (the reference's kp_rope.py; complex form) against
    the reference's src/utils/rope.py apply_rotary_emb(use_real=False); the
    real form is refused."""
    from harp_b200.ops import modules as kp_rope

    R = _load("src/utils/rope.py")
    x = torch.randn(2, 3, 10, 16)
    ang = torch.rand(2, 10, 8) * 6
    f = torch.polar(torch.ones_like(ang), ang)
    torch.testing.assert_close(kp_rope.kp_apply_rotary_emb(x, f, use_real=False),
                               R.apply_rotary_emb(x, f, use_real=False), rtol=0, atol=1e-5)
    with pytest.raises(NotImplementedError):
        kp_rope.kp_apply_rotary_emb(x, f)


def test_metadata():
    """src/utils/metadata.py: normalised vectors, caption text and the inverse
    map (is_print=False; the reference's is_print=True path reads an attribute
    it never sets)."""
    from harp_b200.utils.misc import MetaData

    R = _load("src/utils/metadata.py")
    a, b = R.MetaData(), MetaData()
    for m in ((116.4, 39.9, 0.5, 2019.0), (-70.25, -33.5, 2.0, 0.0), (10.0, 5.0, 0.123456789, 1999.0)):
        torch.testing.assert_close(a.normalize(m), b.normalize(m))
        assert a.text_formatting(m) == b.text_formatting(m)
        n = a.normalize(m).tolist()
        torch.testing.assert_close(a.unnormalize(n), b.unnormalize(n))
        va, ta = a.embedding(m)
        vb, tb = b.embedding(m)
        torch.testing.assert_close(va, vb)
        assert ta == tb


def test_zimage_matches_the_reference_models_own_forward_and_backward():
    """src/models/z_image/standalone_transformer.py (the reference's own Z-Image
    model, plain PyTorch, fp32) loads into harp's model with every key
    matching, and on shared weights the two predict the same images and give
    the same parameter gradients, to the bf16 rounding of harp's GEMM
    outputs.  The batch mixes image sizes and caption lengths that need
    padding."""
    from harp_b200.models import zimage as Z

    R = _load("src/models/z_image/standalone_transformer.py")
    pre = dict(Z.PRESETS["zimage-tiny"])
    torch.manual_seed(0)
    ref = R.ZImageTransformer2DModel(**{k: (list(v) if isinstance(v, tuple) else v) for k, v in pre.items()})
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.05)
    ours = Z.ZImageTransformer2DModel(**pre)
    ours.load_state_dict(ref.state_dict(), strict=True)
    x = [torch.randn(16, 1, 18, 18), torch.randn(16, 1, 16, 12)]
    caps = [torch.randn(20, pre["cap_feat_dim"]), torch.randn(32, pre["cap_feat_dim"])]
    t = torch.rand(2)
    a = ref(x, t, caps).sample
    b = ours(x, t, caps)["sample"]
    w = [torch.randn_like(u) for u in a]
    sum((u * v).sum() for u, v in zip(a, w)).backward()
    sum((u.float() * v).sum() for u, v in zip(b, w)).backward()
    for u, v in zip(a, b):
        assert ((u - v.float()).abs().max() / u.abs().max()).item() < 2e-2
    theirs = dict(ref.named_parameters())
    for n, p in ours.named_parameters():
        g = theirs[n].grad
        err = ((p.grad.float() - g).abs().max() / g.abs().max().clamp_min(1e-12)).item()
        assert err < 5e-2, (n, err)


@pytest.mark.parametrize("with_cond", [False, True])
def test_legacy_token_layout(with_cond):
    """src/models/z_image/base.py (the legacy model's Z_Mixin) against
    harp_b200.models.zimage_legacy.Z_Mixin: padded token runs, position ids and
    pad masks of captions, images and condition images, and unpatchify."""
    from harp_b200.models.zimage_legacy import Z_Mixin

    R = _load("src/models/z_image/base.py")
    ref, ours = R.Z_Mixin(), Z_Mixin()
    torch.manual_seed(0)
    imgs = [torch.randn(16, 1, 18, 18), torch.randn(16, 2, 16, 12)]
    caps = [torch.randn(20, 8), torch.randn(32, 8)]
    conds = [torch.randn(12, 18, 18), torch.randn(12, 16, 12)] if with_cond else None
    a = ref.patchify_and_embed(imgs, caps, 2, 1, conds)
    b = ours.patchify_and_embed(imgs, caps, 2, 1, conds)
    for part_a, part_b in zip(a[:7], b[:7]):
        assert len(part_a) == len(part_b)
        for u, v in zip(part_a, part_b):
            if isinstance(u, torch.Tensor):
                torch.testing.assert_close(v, u, rtol=0, atol=0)
            else:
                assert tuple(u) == tuple(v)
    if with_cond:
        for part_a, part_b in zip(a[7], b[7]):
            for u, v in zip(part_a, part_b):
                torch.testing.assert_close(v, u, rtol=0, atol=0)
    else:
        assert a[7] is None and b[7] is None
    toks = [torch.randn(t.shape[0], 2 * 2 * 1 * 16) for t in a[0]]
    want = ref.unpatchify([t.clone() for t in toks], a[2], 2, 1, 16)
    got = ours.unpatchify([t.clone() for t in toks], b[2], 2, 1, 16)
    for u, v in zip(want, got):
        torch.testing.assert_close(v, u, rtol=0, atol=0)


def _cli_flags(path):
    """{flag: {type, default, action, choices}} of every literal add_argument
    call in a script, read from its syntax tree (the script is not run)."""
    import ast

    flags = {}
    for node in ast.walk(ast.parse(open(path).read())):
        if isinstance(node, ast.Call) and getattr(node.func, "attr", None) == "add_argument":
            names = [a.value for a in node.args if isinstance(a, ast.Constant)]
            if not names:
                continue
            kw = {}
            for k in node.keywords:
                if k.arg in ("type", "default", "action", "choices"):
                    v = k.value
                    kw[k.arg] = ast.literal_eval(v) if isinstance(v, (ast.Constant, ast.List)) else ast.unparse(v)
            flags[names[0]] = kw
    return flags


def test_train_cli_accepts_every_reference_flag():
    """train.py (the reference's, read as text) against harp's train.py: every
    reference flag parses, with the reference's type, default and choices."""
    import sys

    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref_flags = _cli_flags(os.path.join(REF, "train.py"))
    assert len(ref_flags) >= 25
    sys.path.insert(0, here)
    try:
        import train as T
    finally:
        sys.path.remove(here)
    args = vars(T.parse_args([]))
    types = {"str": str, "int": int, "float": float, "bool": bool}
    for flag, kw in ref_flags.items():
        dest = flag.lstrip("-").replace("-", "_")
        assert dest in args, flag
        if "default" in kw:
            assert args[dest] == kw["default"], (flag, args[dest], kw["default"])
        elif kw.get("action") == "store_true":
            assert args[dest] is False, flag
        if kw.get("type") in types and args[dest] is not None:
            assert isinstance(args[dest], types[kw["type"]]), flag
        if "choices" in kw:
            for c in kw["choices"]:
                assert vars(T.parse_args([flag, c]))[dest] == c, (flag, c)


class _FakeAccelerator:
    is_main_process = True

    @staticmethod
    def unwrap_model(m):
        return m


class _LoraModel(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.base = torch.nn.Linear(4, 3)
        self.lora_A = torch.nn.Linear(4, 2, bias=False)
        self.frozen = torch.nn.Linear(3, 3)
        self.frozen.requires_grad_(False)
        self.saved = []

    def save_lora_adapter(self, save_directory, adapter_name):
        self.saved.append((os.path.basename(save_directory), adapter_name))


def test_checkpoint_hooks_and_helpers(tmp_path):
    """src/utils/hook.py and src/utils/utils.py: the accelerate save hooks write
    the same model.safetensors (trainable, non-LoRA tensors) and call the same
    adapter saves; preserve_requires_grad restores the flags; encode_images
    applies the VAE's shift and scale."""
    from safetensors.torch import load_file

    from harp_b200.utils import misc as M

    H = _load("src/utils/hook.py")
    U = _load("src/utils/utils.py")
    torch.manual_seed(0)
    model = _LoraModel()
    for hook_ref, hook_ours, extra in ((H.save_trainable_param_hook, M.save_trainable_param_hook, {}),
                                       (H.save_lora_adapter_hook, M.save_lora_adapter_hook,
                                        {"target_adapters": ["a", "b"]})):
        outs = []
        for i, hook in enumerate((hook_ref, hook_ours)):
            d = tmp_path / f"{hook.__name__}{i}"
            d.mkdir()
            weights = [object()]
            model.saved = []
            hook([model], weights, str(d), _FakeAccelerator(), **extra)
            assert weights == []
            outs.append((load_file(str(d / "model.safetensors")), list(model.saved)))
        (sa, la), (sb, lb) = outs
        assert sorted(sa) == sorted(sb) == ["base.bias", "base.weight"]
        for k in sa:
            assert torch.equal(sa[k], sb[k])
        assert la == lb
    for ctx in (U.preserve_requires_grad, M.preserve_requires_grad):
        with ctx(model):
            model.requires_grad_(False)
            model.frozen.requires_grad_(True)
        assert model.base.weight.requires_grad and not model.frozen.weight.requires_grad

    class _Dist:
        def __init__(self, z):
            self.z = z

        def sample(self):
            return self.z

    class _VAE:
        dtype = torch.float32

        class config:
            shift_factor, scaling_factor = 0.1159, 0.3611

        def encode(self, x):
            return type("Out", (), {"latent_dist": _Dist(x * 2.0)})()

    px = torch.randn(2, 3, 8, 8)
    torch.testing.assert_close(M.encode_images(_VAE(), px, torch.bfloat16),
                               U.encode_images(_VAE(), px, torch.bfloat16), rtol=0, atol=0)


@pytest.mark.parametrize("branches", [0, 1, 2])
def test_sp_token_layout(branches):
    """src/models/z_image/hl_base.py (the SP model's Z_Mixin: one list of
    condition images per branch, branch j on the plane caption + 2 + j)
    against harp's Z_HLMixin, which the SP Z_Transformer inherits."""
    from harp_b200.models.zimage import Z_HLMixin

    R = _load("src/models/z_image/hl_base.py")
    ref, ours = R.Z_Mixin(), Z_HLMixin()
    torch.manual_seed(0)
    imgs = [torch.randn(16, 1, 18, 18), torch.randn(16, 1, 16, 12)]
    caps = [torch.randn(20, 8), torch.randn(32, 8)]
    conds = [[torch.randn(12, 18, 18), torch.randn(12, 16, 12)] for _ in range(branches)] or None
    a = ref.patchify_and_embed(imgs, caps, 2, 1, conds)
    b = ours.patchify_and_embed(imgs, caps, 2, 1, conds)
    for part_a, part_b in zip(a[:7], b[:7]):
        for u, v in zip(part_a, part_b):
            if isinstance(u, torch.Tensor):
                torch.testing.assert_close(v, u, rtol=0, atol=0)
            else:
                assert tuple(u) == tuple(v)
    if conds is None:
        assert a[7] is None and b[7] is None
        return
    assert sorted(a[7]) == sorted(b[7])
    for key in a[7]:
        assert [len(x) for x in a[7][key]] == [len(x) for x in b[7][key]]
        for la, lb in zip(a[7][key], b[7][key]):
            for u, v in zip(la, lb):
                torch.testing.assert_close(v, u, rtol=0, atol=0)


def test_npz_dataset_and_collate(tmp_path):
    """src/datatsets/TiffDataset.py (NpzDataset, custom_collate_fn) against
    harp_b200.utils.data on .npz samples of the reference's format.  That file
    uses json, numpy and torch without importing them; the test supplies the
    three modules to it."""
    import numpy as np

    from harp_b200.utils import data as D

    R = _load("src/datatsets/TiffDataset.py")
    R.json, R.np, R.torch = json, np, torch
    rng = np.random.default_rng(0)
    files = []
    for i, L in enumerate((20, 32, 7)):
        f = tmp_path / f"s{i}.npz"
        np.savez(f, norm_metadata=rng.random(4).astype(np.float32),
                 prompt_embeds=rng.random((L, 16)).astype(np.float32),
                 latent_image=rng.random((16, 8, 8)).astype(np.float32),
                 cond=rng.random((12, 8, 8)).astype(np.float32))
        files.append(str(f))
    index = tmp_path / "index.json"
    index.write_text(json.dumps(files))
    a, b = R.NpzDataset(str(index)), D.NpzDataset(str(index))
    assert len(a) == len(b) == 3
    for i in range(3):
        for k, v in a[i].items():
            assert np.array_equal(v, b[i][k]), k
    ca, cb = R.custom_collate_fn([a[i] for i in range(3)]), D.custom_collate_fn([b[i] for i in range(3)])
    assert sorted(ca) == sorted(cb)
    torch.testing.assert_close(ca["norm_metadata"], cb["norm_metadata"], rtol=0, atol=0)
    torch.testing.assert_close(ca["latent_image"], cb["latent_image"], rtol=0, atol=0)
    for u, v in zip(ca["prompt_embeds"], cb["prompt_embeds"]):
        torch.testing.assert_close(u, v, rtol=0, atol=0)
    assert len(ca["cond"]) == len(cb["cond"]) == 1
    torch.testing.assert_close(ca["cond"][0], cb["cond"][0], rtol=0, atol=0)


def test_broadcasting_autograd_ops():
    """async_rt/async_ops.py:55-122 (MyMul, MyAdd; the file's other ops call
    the reference's compiled library) against harp's, with broadcasting and a
    Python-number operand."""
    from harp_b200.runtime import async_compat as O

    R = _load("async_rt/async_ops.py")
    torch.manual_seed(0)
    a0, b0 = torch.randn(4, 1, 5), torch.randn(3, 5)
    for fn in ("MyMul", "MyAdd"):
        outs = []
        for mod in (R, O):
            a, b = a0.clone().requires_grad_(True), b0.clone().requires_grad_(True)
            y = getattr(mod, fn).apply(a, b)
            y.pow(2).sum().backward()
            outs.append((y.detach(), a.grad, b.grad))
        for u, v in zip(*outs):
            torch.testing.assert_close(v, u, rtol=0, atol=0)
    outs = []
    for mod in (R, O):
        b = b0.clone().requires_grad_(True)
        y = mod.MyAdd.apply(1.5, b)
        (y * b0).sum().backward()
        outs.append((y.detach(), b.grad))
    for u, v in zip(*outs):
        torch.testing.assert_close(v, u, rtol=0, atol=0)


def test_train_cli_on_the_reference_sample_data(tmp_path):
    """harp's train.py reads the reference's shipped samples (data/index.json,
    whose entries are "HARP/data/..." paths) and trains a small Z-Image with
    their shapes (caption features 2560 wide, 16 x 64 x 64 latents, 192-channel
    condition images, 4 metadata values) for two steps, with finite losses."""
    import subprocess
    import sys

    from harp_b200.utils.data import NpzDataset

    index = os.path.join(REF, "data", "index.json")
    assert len(NpzDataset(index)) == len(json.load(open(index)))
    cfg_dir = tmp_path / "cfg" / "transformer"
    cfg_dir.mkdir(parents=True)
    (cfg_dir / "config.json").write_text(json.dumps({
        "all_patch_size": [2], "all_f_patch_size": [1], "in_channels": 16, "dim": 64, "n_layers": 1,
        "n_refiner_layers": 1, "n_heads": 2, "n_kv_heads": 2, "cap_feat_dim": 2560, "axes_dims": [8, 12, 12],
        "axes_lens": [2048, 64, 64]}))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    work = tmp_path / "w"
    cmd = [sys.executable, os.path.join(root, "train.py"), "--model", "zimage-tiny", "--pretrained_model_name_or_path",
           str(tmp_path / "cfg"), "--data_root", index, "--max_train_steps", "2", "--train_batch_size", "1",
           "--sp_size", "1", "--work_dir", str(work), "--lr_warmup_steps", "1", "--checkpointing_steps", "100"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=str(tmp_path),
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-3000:]
    (run,) = os.listdir(work)
    rows = [json.loads(line) for line in open(work / run / "metrics.jsonl") if line.strip()]
    losses = [row["step_loss"] for row in rows if "step_loss" in row]
    assert len(losses) == 2 and all(math.isfinite(v) for v in losses)


def _load_reference_inference(monkeypatch):
    """src/utils/inference.py imports diffusers (not needed for latent output);
    stand-ins for the names it imports let the module load."""
    import sys
    import types

    def randn_tensor(shape, generator=None, device=None, dtype=None):
        return torch.randn(shape, generator=generator, dtype=dtype).to(device)

    mods = {n: types.ModuleType(n) for n in ("diffusers", "diffusers.utils", "diffusers.utils.torch_utils",
                                             "diffusers.image_processor", "diffusers.pipelines",
                                             "diffusers.pipelines.z_image",
                                             "diffusers.pipelines.z_image.pipeline_output")}
    mods["diffusers.utils.torch_utils"].randn_tensor = randn_tensor
    mods["diffusers.image_processor"].VaeImageProcessor = object
    for n in ("ZImageTransformer2DModel", "AutoencoderKL", "FlowMatchEulerDiscreteScheduler"):
        setattr(mods["diffusers"], n, object)
    mods["diffusers.pipelines.z_image.pipeline_output"].ZImagePipelineOutput = dict
    for n, m in mods.items():
        monkeypatch.setitem(sys.modules, n, m)
    return _load("src/utils/inference.py")


@pytest.mark.parametrize("cfg", [None, dict(guidance_scale=4.0, cfg_truncation=0.6, cfg_normalization=1.2)])
def test_sampling_loop_matches_the_reference(monkeypatch, cfg):
    """src/utils/inference.py batch_image_inference (the reference's sampling
    loop: shifted flow-match grid, classifier-free guidance with truncation
    and renormalisation, Euler steps) against harp_b200.inference's, with the
    same model (harp's SP Z-Image, which the reference loop calls with its own
    convention: transformer(x=..., t=..., text_embedding=..., return_dict=False)[0]
    gives one [C, 1, H, W] per sample) and harp's scheduler in both: the same
    final latents."""
    from harp_b200 import inference as HI
    from harp_b200.models import zimage as Z
    from harp_b200.utils.diffusion import FlowMatchEulerDiscreteScheduler

    R = _load_reference_inference(monkeypatch)
    torch.manual_seed(0)
    pre = Z.PRESETS["zimage-tiny"]
    model = Z.Z_Transformer(Z.ZImageTransformer2DModel(**pre))
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0, 0.05)
    model = model.bfloat16()

    g = torch.Generator().manual_seed(1)
    lat = torch.randn(2, 16, 16, 16, generator=g).bfloat16()
    pos = [torch.randn(32, pre["cap_feat_dim"], generator=g).bfloat16() for _ in range(2)]
    neg = [torch.randn(32, pre["cap_feat_dim"], generator=g).bfloat16() for _ in range(2)] if cfg else None
    kw = dict(prompt_embeds=pos, negative_prompt_embeds=neg, num_inference_steps=6, output_type="latent",
              return_dict=False, initial_latents=lat.clone(), vae_scale_factor=8, **(cfg or {}))

    def scheduler():
        return FlowMatchEulerDiscreteScheduler(shift=3.0, use_dynamic_shifting=True)

    want = R.batch_image_inference(model, None, scheduler(), None, **kw)[0]
    got = HI.batch_image_inference(model, None, scheduler(), None, **kw)[0]
    assert got.dtype == want.dtype == torch.bfloat16
    assert ((got.float() - want.float()).norm() / want.float().norm()).item() < 5e-3


@pytest.mark.parametrize("max_nodes", [None, 2])
def test_mpi_rankfile_matches_the_reference(tmp_path, capsys, max_nodes):
    """gen_rankfile/gen_rankfile.py (the reference's OpenMPI rankfile for its
    16-rank, 608-core, two-socket nodes) against harp_b200.launch's
    generate_rankfile(fmt="mpi") with those parameters: the same lines, nodes
    in natural order, truncated to max_nodes."""
    from harp_b200.launch import generate_rankfile

    R = _load("gen_rankfile/gen_rankfile.py")
    hosts = ["node10", "node2", "node1", "gpu-a3"]
    hostfile = tmp_path / "nodes.txt"
    hostfile.write_text("\n".join(f"{h} slots=16" for h in hosts) + "\n")
    R.generate_cpuset_rankfile(str(hostfile), max_nodes=max_nodes)
    want = capsys.readouterr().out.split("\n")
    want = [line for line in want if line]
    got = generate_rankfile(hosts, ranks_per_node=16, max_nodes=max_nodes, cores_per_node=608, fmt="mpi", sockets=2)
    assert got == want
