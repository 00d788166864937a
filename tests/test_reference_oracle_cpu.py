"""Oracle tests against the reference's own pure-PyTorch modules.

The reference project's root is read from HARP_REFERENCE_DIR; every test here
is skipped when it is unset.  Only files that import nothing but torch (and the
standard library) are loaded, one at a time with importlib, so none of the
reference's compiled extensions are needed.  Each test runs the reference's
function and harp's on the same inputs.
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
    ours = RopeEmbedder(256.0, dims, lens)
    ids = torch.stack([torch.randint(0, n, (300,)) for n in lens], -1).int()
    torch.testing.assert_close(ours.complex(ids), ref(ids), rtol=0, atol=2e-6)


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
