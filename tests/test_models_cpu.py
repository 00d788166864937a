"""Model-level numerics on CPU: the fused DiT block (hand-written forward and
backward over harp_b200.ops) against plain fp32 autograd of the same math, and
forward/backward of every model family (DiT, Z-Image, MMDiT, Flux)."""
import math
import os

import pytest
import torch
import torch.nn.functional as F

from harp_b200.models import dit as D
from harp_b200.models import mmdit as M
from harp_b200.models import zimage as Z
from harp_b200.parallel.sequence import SPContext


def _rms(x, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def _rope(x, freqs):
    # x [B, S, H, Dh]; freqs [S, Dh/2, 2] (cos, sin) of adjacent pairs
    cos, sin = freqs[None, :, None, :, 0], freqs[None, :, None, :, 1]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], -1).flatten(-2)


def reference_block(x, c_silu, freqs, p, cfg):
    """Plain fp32 DiT block: adaLN-zero, RMSNorm+modulate, QK-norm, RoPE,
    attention, gated residual, SwiGLU MLP, gated residual."""
    B, S, Dm = x.shape
    H, Dh = cfg.heads, cfg.head_dim
    mod = (c_silu @ p["ada_w"].T + p["ada_b"]).unsqueeze(1)
    sh1, sc1, g1, sh2, sc2, g2 = mod.chunk(6, -1)
    h1 = _rms(x, cfg.norm_eps) * (1 + sc1) + sh1
    qkv = h1 @ p["qkv_w"].T + p["qkv_b"]
    q, k, v = qkv.chunk(3, -1)
    q = _rms(q.view(B, S, H, Dh), 1e-6) * p["qn"]
    k = _rms(k.view(B, S, H, Dh), 1e-6) * p["kn"]
    q, k = _rope(q, freqs), _rope(k, freqs)
    v = v.view(B, S, H, Dh)
    att = torch.softmax(torch.einsum("bshd,bthd->bhst", q, k) / math.sqrt(Dh), -1)
    o = torch.einsum("bhst,bthd->bshd", att, v).reshape(B, S, Dm)
    x1 = x + g1 * (o @ p["proj_w"].T + p["proj_b"])
    h2 = _rms(x1, cfg.norm_eps) * (1 + sc2) + sh2
    m = F.silu(h2 @ p["w1"].T) * (h2 @ p["w3"].T)
    return x1 + g2 * (m @ p["w2"].T + p["w2_b"])


def test_dit_block_forward_backward_matches_fp32_reference():
    torch.manual_seed(0)
    cfg = D.DiTConfig(in_channels=4, hidden=64, depth=1, heads=2, mlp_ratio=2.0, text_dim=32, axes_dims=(8, 12, 12))
    blk = D.DiTBlock(cfg, 0)
    with torch.no_grad():
        for prm in blk.parameters():
            prm.copy_(torch.randn_like(prm) * 0.2)
    blk = blk.to(torch.bfloat16)  # the harp ops compute in bf16 with fp32 accumulation
    B, S = 2, 24
    x = torch.randn(B, S, cfg.hidden).bfloat16().requires_grad_(True)
    c = torch.randn(B, cfg.hidden).bfloat16().requires_grad_(True)
    freqs = D.rope_freqs(D.joint_positions(4, 4, 8), cfg.axes_dims, cfg.rope_theta)
    y = blk(x, c, freqs, SPContext())
    gy = torch.randn_like(y)
    y.backward(gy)
    gy = gy.float()

    a, m = blk.attn, blk.mlp
    names = {"ada_w": blk.adaLN_modulation[1].weight, "ada_b": blk.adaLN_modulation[1].bias,
             "qkv_w": a.qkv.weight, "qkv_b": a.qkv.bias, "qn": a.q_norm.weight, "kn": a.k_norm.weight,
             "proj_w": a.proj.weight, "proj_b": a.proj.bias, "w1": m.w1.weight, "w3": m.w3.weight,
             "w2": m.w2.weight, "w2_b": m.w2.bias}
    ref_p = {k: v.detach().float().clone().requires_grad_(True) for k, v in names.items()}
    xr = x.detach().float().clone().requires_grad_(True)
    cr = c.detach().float().clone().requires_grad_(True)
    yr = reference_block(xr, cr, freqs, ref_p, cfg)
    yr.backward(gy)

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm().clamp_min(1e-12)).item()

    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 2e-2
    assert rel(c.grad, cr.grad) < 2e-2
    for k, prm in names.items():
        assert rel(prm.grad, ref_p[k].grad) < 2e-2, (k, rel(prm.grad, ref_p[k].grad))


@pytest.mark.parametrize("name", ["tiny"])
def test_dit_model_loss_and_all_grads(name):
    model = D.DiT(D.PRESETS[name])
    model.initialize_weights(0)
    model = model.to(torch.bfloat16)
    lat = torch.randn(2, model.cfg.in_channels, 16, 16).bfloat16()
    text = torch.randn(2, 16, model.cfg.text_dim).bfloat16()
    loss = D.flow_matching_loss_local(model, lat, torch.randn_like(lat), text, torch.rand(2), SPContext())
    loss.backward()
    assert torch.isfinite(loss)
    # adaLN-zero: at init the blocks are the identity, so the final layer and
    # the embedders carry the loss; every parameter still receives a gradient
    assert all(p.grad is not None for p in model.parameters())


@pytest.mark.parametrize("name", ["mmdit-tiny", "flux-tiny"])
def test_mmdit_family_forward_backward(name):
    torch.manual_seed(0)
    model = M.MMDiT(M.PRESETS[name])
    model.initialize_weights(1)
    with torch.no_grad():  # leave adaLN-zero so every branch carries gradient
        for n, prm in model.named_parameters():
            if ".mod." in n:
                prm.normal_(0, 0.02)
    model = model.to(torch.bfloat16)
    lat = torch.randn(2, 16, 16, 16).bfloat16()
    text = torch.randn(2, 32, model.cfg.text_dim).bfloat16()
    loss = M.mmdit_loss_local(model, lat, torch.randn_like(lat), text, torch.rand(2), SPContext())
    loss.backward()
    assert torch.isfinite(loss)
    missing = [n for n, p in model.named_parameters() if p.grad is None or not torch.isfinite(p.grad.float()).all()]
    assert not missing, missing
    # the queries of a pre-only text stream feed outputs that are never read
    pre_only = {f"double_blocks.{i}.txt.norm.query_norm" for i, b in enumerate(model.double_blocks) if b.txt.pre_only}
    nz = [n for n, p in model.named_parameters() if p.grad.float().abs().sum() == 0 and n not in pre_only]
    assert not nz, nz


def test_zimage_forward_backward_and_state_dict_layout():
    torch.manual_seed(0)
    base = Z.ZImageTransformer2DModel(**Z.PRESETS["zimage-tiny"])
    model = Z.Z_Transformer(base, num_metadata=4, use_cond=True).to(torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0, 0.02)
    lat = torch.randn(2, 16, 16, 16).bfloat16()
    text = torch.randn(2, 32, Z.PRESETS["zimage-tiny"]["cap_feat_dim"]).bfloat16()
    meta = torch.rand(2, 4).bfloat16()
    cond = [torch.randn(2, 192, 16, 16).bfloat16()]
    loss = Z.zimage_loss_local(model, lat, torch.randn_like(lat), text, torch.rand(2), SPContext(), metadata=meta,
                               cond=cond)
    loss.backward()
    assert torch.isfinite(loss)
    keys = set(model.state_dict().keys())
    # names follow the reference's checkpoint layout (diffusers Z-Image + cond branch)
    for k in ("cond_pad_token", "cond_refiner_1.0.attention.attn.to_q.weight",
              "cond_refiner_1.0.z_block.feed_forward.w1.weight"):
        assert k in keys, k
    used = [n for n, p in model.named_parameters() if p.grad is not None]
    assert any(n.startswith("cond_refiner_1") for n in used)


def test_rope_tables():
    pos = D.joint_positions(2, 3, 4)
    assert pos.shape == (10, 3)
    assert (pos[:6, 0] == 5).all() and (pos[6:, 0] == torch.arange(1, 5)).all()
    f = D.rope_freqs(pos, (4, 6, 6), 10000.0)
    assert f.shape == (10, 8, 2)
    torch.testing.assert_close(f[..., 0].pow(2) + f[..., 1].pow(2), torch.ones(10, 8))


def test_cfg_inference_runs_for_every_family():
    from harp_b200 import inference as I
    from harp_b200.utils.diffusion import FlowMatchEulerDiscreteScheduler as FS

    torch.manual_seed(0)
    dit = D.DiT(D.PRESETS["tiny"])
    dit.initialize_weights(0)
    dit = dit.bfloat16()
    pe = [torch.randn(16, dit.cfg.text_dim).bfloat16() for _ in range(2)]
    ne = [torch.zeros(16, dit.cfg.text_dim).bfloat16() for _ in range(2)]
    out = I.batch_image_inference(dit, None, FS(use_dynamic_shifting=True), None, pe, ne, height=128, width=128,
                                  num_inference_steps=3, guidance_scale=3.0, cfg_normalization=1.5,
                                  generator=torch.Generator().manual_seed(0), in_channels=dit.cfg.in_channels)
    assert out["images"].shape == (2, dit.cfg.in_channels, 16, 16)
    assert torch.isfinite(out["images"].float()).all()
    # zero velocity everywhere -> the Euler sampler returns its starting noise
    with torch.no_grad():
        dit.final_layer.linear.weight.zero_()
        dit.final_layer.linear.bias.zero_()
    x0 = torch.randn(1, dit.cfg.in_channels, 16, 16).bfloat16()
    out = I.batch_image_inference(dit, None, FS(), None, pe[:1], None, num_inference_steps=2, initial_latents=x0,
                                  return_dict=False)[0]
    assert torch.equal(out, x0)
    zm = Z.Z_Transformer(Z.ZImageTransformer2DModel(**Z.PRESETS["zimage-tiny"]), num_metadata=4, use_cond=False)
    zm = zm.bfloat16()
    with torch.no_grad():
        for p in zm.parameters():
            p.normal_(0, 0.02)
    pz = [torch.randn(16, 64).bfloat16() for _ in range(2)]
    out = I.batch_image_inference(zm, None, FS(), None, pz, pz, height=128, width=128, num_inference_steps=2,
                                  generator=torch.Generator().manual_seed(0), in_channels=16,
                                  metadata=torch.rand(2, 4).bfloat16())
    assert out["images"].shape == (2, 16, 16, 16)


def test_scheduler_inference_grid():
    from harp_b200.utils.diffusion import FlowMatchEulerDiscreteScheduler as FS

    s = FS(shift=3.0)
    s.sigma_min = 0.0
    s.set_timesteps(4)
    assert s.sigmas.shape == (5,) and s.sigmas[-1] == 0 and s.sigmas[0] == pytest.approx(1.0)
    d = FS(use_dynamic_shifting=True)
    d.set_timesteps(4, mu=1.0)
    assert torch.all(d.sigmas[:-1][1:] < d.sigmas[:-1][:-1])


def test_ring_attention_ops_match_sdpa():
    from harp_b200.ops import ring_ops

    ring_ops.set_sp_context(None)
    g = torch.Generator().manual_seed(3)
    B, T, H, D = 1, 24, 2, 16
    q, k, v = (torch.randn(B, T, H, D, generator=g).bfloat16().transpose(1, 2).requires_grad_(True) for _ in range(3))
    out = ring_ops.CPURingAttention.apply(q, k, v, 1)
    do = torch.randn_like(out)
    out.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qr, kr, vr)
    ref.backward(do.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    for a, b in ((q, qr), (k, kr), (v, vr)):
        torch.testing.assert_close(a.grad.float(), b.grad, rtol=5e-2, atol=5e-2)
    with pytest.raises(RuntimeError):
        ring_ops.CPURingAttention.apply(q, k, v, 2)


def test_ring_attention_ops_any_scale_and_saved_statistics():
    """The op pair with a non-default softmax scale; the backward takes the
    LSE (m_i, l_i) and D from its arguments."""
    from harp_b200.ops import ring_ops

    ring_ops.set_sp_context(None)
    g = torch.Generator().manual_seed(5)
    B, T, H, D = 2, 40, 3, 16
    scale = 0.37
    q, k, v = (torch.randn(B, T, H, D, generator=g).bfloat16().transpose(1, 2) for _ in range(3))
    out = torch.zeros(B, H, T, D)
    m_i = torch.empty(B, H, T, 1, dtype=torch.bfloat16)
    l_i = torch.empty(B, H, T, 1)
    torch.ops.ring_attention_ops.ring_attention_forward(q, k, v, out, m_i, l_i, 1, scale)
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qr, kr, vr, scale=scale)
    torch.testing.assert_close(out, ref.detach(), rtol=2e-2, atol=2e-2)
    do = torch.randn(B, H, T, D, generator=g).bfloat16()
    ref.backward(do.float())
    Dt = (do.float() * out).sum(-1, keepdim=True)
    gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    torch.ops.ring_attention_ops.ring_attention_backward(q, gq, k, gk, v, gv, do, m_i, l_i, Dt, 1, scale)
    for a, b in ((gq, qr), (gk, kr), (gv, vr)):
        torch.testing.assert_close(a.float(), b.grad, rtol=5e-2, atol=5e-2)


def test_timestep_embeddings_closed_form():
    from harp_b200.models import embedding as E

    t = torch.tensor([0.0, 1.0, 250.5])
    e = E.get_timestep_embedding(t, 9, flip_sin_to_cos=True, downscale_freq_shift=0)
    half = 4
    f = torch.exp(-math.log(10000) * torch.arange(half) / half)
    torch.testing.assert_close(e[:, :half], torch.cos(t[:, None] * f))
    torch.testing.assert_close(e[:, half:2 * half], torch.sin(t[:, None] * f))
    assert e.shape == (3, 9) and torch.all(e[:, -1] == 0)
    torch.testing.assert_close(E.Timesteps(8, False, 1)(t), E.get_timestep_embedding(t, 8))
    te = E.TimestepEmbedding(8, 16, out_dim=4, cond_proj_dim=3)
    assert te(torch.randn(2, 8), torch.randn(2, 3)).shape == (2, 4)
    emb = E.TimestepEmbedder(32, frequency_embedding_size=16)
    assert {n for n, _ in emb.named_parameters()} == {"mlp.0.weight", "mlp.0.bias", "mlp.2.weight", "mlp.2.bias"}
    assert emb(t).shape == (3, 32)


def test_zimage_legacy_matches_base_and_groups_variable_sizes():
    """The legacy (non-SP, variable-size) Z-Image wrapper: on equal-size samples
    without padding it gives the base model's output; a batch of mixed image
    sizes and caption lengths gives each sample's output on its own; the LoRA
    target names resolve to modules."""
    import copy

    from harp_b200.models import zimage_legacy as ZL

    torch.manual_seed(0)
    pre = Z.PRESETS["zimage-tiny"]
    base = Z.ZImageTransformer2DModel(**pre)
    with torch.no_grad():
        for p in base.parameters():
            p.normal_(0, 0.05)
    base = base.bfloat16()
    ref_base = copy.deepcopy(base)
    model = ZL.Z_Transformer(base, num_metadata=0, use_cond=True)
    cdim = pre["cap_feat_dim"]
    x = [torch.randn(16, 1, 16, 16).bfloat16() for _ in range(2)]
    t = torch.rand(2)
    caps = [torch.randn(32, cdim).bfloat16() for _ in range(2)]
    with torch.no_grad():
        want = ref_base(x, t, caps)["sample"]
        got = model(x, t, caps)["sample"]
    for a, b in zip(got, want):
        assert a.shape == b.shape == (16, 1, 16, 16)
        torch.testing.assert_close(a.float(), b.float(), rtol=0, atol=0)

    # mixed sizes: 16x16 and 12x20 latents (60 tokens -> padded to 64), captions of 20, 45, 20 tokens
    xs = [torch.randn(16, 1, 16, 16).bfloat16(), torch.randn(16, 1, 12, 20).bfloat16(),
          torch.randn(16, 1, 16, 16).bfloat16()]
    ts = torch.rand(3)
    cps = [torch.randn(20, cdim).bfloat16(), torch.randn(45, cdim).bfloat16(), torch.randn(20, cdim).bfloat16()]
    conds = [torch.randn(192, 16, 16).bfloat16(), torch.randn(192, 12, 20).bfloat16(),
             torch.randn(192, 16, 16).bfloat16()]
    with torch.no_grad():
        batch = model(xs, ts, cps, cond_list=conds)["sample"]
        for i in range(3):
            one = model([xs[i]], ts[i:i + 1], [cps[i]], cond_list=[conds[i]])["sample"][0]
            assert batch[i].shape == xs[i].shape
            torch.testing.assert_close(batch[i].float(), one.float(), rtol=0, atol=0)
    # padded caption tokens take the learned pad token: changing it changes the output
    with torch.no_grad():
        model.z_transformer.cap_pad_token.add_(1.0)
        moved = model([xs[0]], ts[:1], [cps[0]], cond_list=[conds[0]])["sample"][0]
    assert not torch.equal(moved, batch[0])

    out = model(xs[:2], ts[:2], cps[:2], cond_list=conds[:2])["sample"]
    sum(o.float().square().mean() for o in out).backward()
    assert model.cond_refiner[0].z_block.feed_forward.w1.weight.grad is not None
    mods = dict(model.named_modules())
    names = (model.get_noise_lora_branch() + model.get_context_lora_branch() + model.get_main_lora_branch())
    assert names and all(n in mods for n in names), [n for n in names if n not in mods]
    assert model.switch_cond_branch_grad(False) > 0
    assert not model.cond_embedder.weight.requires_grad


def test_zimage_compat_residuals_single_vs_joint():
    """harp_block_compat: without modulation Z_SingleBlock keeps the residual
    (x + norm2(ffn(norm1(x)))) and Z_JointBlock replaces it (h + norm2(h))."""
    import copy

    torch.manual_seed(0)
    blk = Z.ZImageTransformerBlock(0, 64, 2, 2, 1e-5, True, modulation=False)
    single = Z.Z_SingleBlock(copy.deepcopy(blk), 1, True)
    joint = Z.Z_JointBlock(copy.deepcopy(blk), 1, True)
    x = torch.randn(1, 32, 64)
    ang = torch.rand(32, 16) * 3
    freqs = torch.stack([ang.cos(), ang.sin()], -1)
    with torch.no_grad():
        ys = single(x, None, freqs)
        yj = joint(x, None, freqs)
        zb = single.z_block
        a = x + zb.attention_norm2(single.attention(zb.attention_norm1(x), freqs, SPContext()))
        h = zb.feed_forward(zb.ffn_norm1(a))
    torch.testing.assert_close(ys, a + zb.ffn_norm2(h))
    torch.testing.assert_close(yj, h + zb.ffn_norm2(h))


def test_mmdit_reports_parameters_a_rank_does_not_use():
    """A sequence-parallel rank that holds no text tokens reports the text
    stream's and the text embedder's parameters as gradient-complete during the
    forward (their zeroed slots get nothing), so an overlapped bucketed gradient
    sync does not wait for them; the parameters it uses are not reported."""
    torch.manual_seed(0)
    cfg = M.PRESETS["flux-tiny"]
    model = M.MMDiT(cfg)
    model.initialize_weights(0)
    seen = []
    for p in model.parameters():
        p._harp_grad_ready = seen.append
    B, n = 1, 48
    blk = model.double_blocks[0]
    with torch.no_grad():  # this rank's 48 tokens are all image tokens
        blk(torch.zeros(B, n, cfg.hidden), n, torch.zeros(B, cfg.hidden), torch.zeros(n, cfg.head_dim // 2, 2),
            SPContext())
    ids = {id(p) for p in seen}
    assert {id(p) for p in blk.txt.parameters()} <= ids
    assert not ({id(p) for p in blk.img.parameters()} & ids)
    seen.clear()
    with torch.no_grad():  # no text tokens at all: the text embedder gets no gradient
        model.forward_local(torch.randn(B, 64, cfg.patch_dim), torch.randn(B, 0, cfg.text_dim), torch.rand(B), 8, 8,
                            SPContext())
    ids = {id(p) for p in seen}
    assert {id(p) for p in model.txt_in.parameters()} <= ids
    assert not ({id(p) for p in model.img_in.parameters()} & ids)


def test_ulysses_dkv_push_addresses_match_the_remap():
    """The attention backward's dK/dV push arguments for the Ulysses layout
    (uly_dkv_push) put every element where the head-to-sequence remap puts it:
    the kernel's destination (base[c] + (b*chunk + s)*ld + hn*Dh (+vcol), as in
    dkv_dst_row of attention_sm100.cu) against the remap's (base[c] +
    (b*S + s)*ld + p*pcol + (rank*Hn + hn)*Dh, uly_remap_kernel in ulysses.cu)."""
    from harp_b200.parallel.nvlink import uly_dkv_push

    for W, H, Dh, S, B in ((2, 16, 72, 64, 2), (8, 16, 72, 32, 1), (4, 24, 128, 48, 2)):
        bases = [(c + 1) << 32 for c in range(W)]
        HD, Hn = H * Dh, H // W
        for rank in range(W):
            a = uly_dkv_push(bases, rank, H, Dh, S)
            assert a["chunk"] * W == W * S and a["ld"] % 8 == 0 and a["vcol"] % 8 == 0
            for b in range(B):
                for key in (0, S - 1, S, W * S - 1):
                    c, s = key // a["chunk"], key % a["chunk"]
                    for hn in (0, Hn - 1):
                        for is_v, part in ((False, 1), (True, 2)):
                            kern = a["bases"][c] + 2 * ((b * a["chunk"] + s) * a["ld"] + (a["vcol"] if is_v else 0)
                                                        + hn * Dh)
                            remap = bases[c] + 2 * ((b * S + s) * 3 * HD + part * HD + (rank * Hn + hn) * Dh)
                            assert kern == remap, (W, rank, b, key, hn, is_v)
                            assert kern % 16 == 0


@pytest.mark.parametrize("hw,L", [(16, 32), (18, 20)])
def test_zimage_sp_wrapper_matches_base_model(hw, L):
    """The reference never compares its SP wrapper with the base model; here the
    wrapper's forward (one rank, no condition branch or metadata) gives the base
    ZImageTransformer2DModel's prediction on the same weights, also when the
    image and caption runs need pad tokens (18 x 18: 81 image tokens)."""
    import copy

    torch.manual_seed(0)
    pre = Z.PRESETS["zimage-tiny"]
    base = Z.ZImageTransformer2DModel(**pre)
    with torch.no_grad():
        for p in base.parameters():
            p.normal_(0, 0.05)
    base = base.bfloat16()
    ref_base = copy.deepcopy(base)
    model = Z.Z_Transformer(base, num_metadata=0, use_cond=False)
    x = [torch.randn(16, 1, hw, hw).bfloat16() for _ in range(2)]
    t = torch.rand(2)
    caps = [torch.randn(L, pre["cap_feat_dim"]).bfloat16() for _ in range(2)]
    with torch.no_grad():
        want = ref_base(x, t, caps)["sample"]
        pred, lo, hi = model.forward_local(x, t, caps, sp=SPContext())
    assert (lo, hi) == (0, (hw // 2) ** 2)
    with torch.no_grad():  # the reference's output contract: one [C, F, H, W] per sample
        full = model(x, t, caps, return_dict=False)[0]
    for u, v in zip(full, want):
        torch.testing.assert_close(u, v, rtol=0, atol=0)
    want_tok = torch.stack(ref_base.patchify([w.float() for w in want], 2, 1)[0])
    torch.testing.assert_close(pred.float(), want_tok, rtol=0, atol=0)


@pytest.mark.parametrize("name", ["dit-xl-2", "mmdit-2b", "flux-12b"])
def test_comparison_arm_models_have_the_same_parameters(name):
    """The NCCL + cuBLAS/SDPA comparison arm (baseline/) builds the same models:
    equal parameter counts for the benchmark configurations (built on the meta
    device, no memory)."""
    import os
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline"))
    if name.startswith("dit"):
        import dit_baseline as B

        with torch.device("meta"):
            ours, theirs = D.DiT(D.PRESETS[name]), B.BaselineDiT(D.PRESETS[name])
    else:
        import mmdit_baseline as B

        with torch.device("meta"):
            ours, theirs = M.MMDiT(M.PRESETS[name]), B.BaselineMMDiT(M.PRESETS[name])
    assert sum(p.numel() for p in ours.parameters()) == sum(p.numel() for p in theirs.parameters())


def _baseline_module(name):
    import os
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline"))
    import importlib

    return importlib.import_module(name)


def _baseline_name(n):
    """harp parameter name -> the comparison arm's name for the same weight."""
    for a, b in (("final_layer.adaLN_modulation.1", "final_ada"), ("final_layer.linear", "final"),
                 ("t_embedder.mlp.0", "t1"), ("t_embedder.mlp.2", "t2"), ("time_in.mlp.0", "t1"),
                 ("time_in.mlp.2", "t2"), ("adaLN_modulation.1", "ada"), (".mod.1.", ".mod."),
                 ("norm.query_norm", "q_norm.weight"), ("norm.key_norm", "k_norm.weight"), ("attn.", ""),
                 ("mlp.", "")):
        n = n.replace(a, b)
    return n


@pytest.mark.parametrize("name", ["tiny", "flux-tiny", "mmdit-tiny"])
def test_comparison_arm_computes_the_same_function(name):
    """Loaded with harp's weights, the comparison arm's model (stock PyTorch)
    predicts what harp's model predicts, to bf16 rounding: the benchmarks
    compare two implementations of one model, not two models."""
    torch.manual_seed(0)
    if name == "tiny":
        B_ = _baseline_module("dit_baseline")
        cfg = D.PRESETS[name]
        ours, theirs = D.DiT(cfg), B_.BaselineDiT(cfg)
    else:
        B_ = _baseline_module("mmdit_baseline")
        cfg = M.PRESETS[name]
        ours, theirs = M.MMDiT(cfg), B_.BaselineMMDiT(cfg)
    ours.initialize_weights(0)
    with torch.no_grad():  # the zero-initialised modulation and output layers get some signal
        for n, p in ours.named_parameters():
            if ".mod." in n or "adaLN" in n or "final" in n:
                p.normal_(0, 0.02)
    ours, theirs = ours.bfloat16(), theirs.bfloat16()
    dst = dict(theirs.named_parameters())
    with torch.no_grad():
        for n, p in ours.named_parameters():
            dst[_baseline_name(n)].copy_(p)
    g = torch.Generator().manual_seed(1)
    lat = torch.randn(2, cfg.in_channels, 16, 16, generator=g).bfloat16()
    text = torch.randn(2, 16, cfg.text_dim, generator=g).bfloat16()
    t = torch.rand(2, generator=g)
    x = ours.patchify(lat)
    with torch.no_grad():
        a, _, _ = ours.forward_local(x, text, t, 8, 8, SPContext())
        b, _, _ = theirs.forward_local(x, text, t, 8, 8, None, 1, 0) if name == "tiny" else \
            theirs(x, text, t, 8, 8, None, 1, 0)
    err = ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
    assert err < 2e-2, err


def test_zimage_variable_sizes_and_caption_lengths():
    """Samples of different image sizes and caption lengths (none a multiple of
    32 tokens) in one batch: each prediction equals that sample run alone, and
    the learned pad tokens receive gradients (they are attended to)."""
    torch.manual_seed(0)
    pre = Z.PRESETS["zimage-tiny"]
    model = Z.ZImageTransformer2DModel(**pre)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0, 0.05)
    x = [torch.randn(16, 1, 18, 18), torch.randn(16, 1, 16, 12), torch.randn(16, 1, 18, 18)]
    caps = [torch.randn(n, pre["cap_feat_dim"]) for n in (20, 32, 7)]
    t = torch.rand(3)
    out = model(x, t, caps)["sample"]
    assert [tuple(o.shape) for o in out] == [tuple(v.shape) for v in x]
    with torch.no_grad():
        for i in range(3):
            alone = model([x[i]], t[i:i + 1], [caps[i]])["sample"][0]
            torch.testing.assert_close(out[i], alone, rtol=0, atol=0)
    sum(o.float().pow(2).mean() for o in out).backward()
    assert model.x_pad_token.grad.abs().max() > 0 and model.cap_pad_token.grad.abs().max() > 0



def test_zimage_sp_wrapper_parameter_groups():
    """The SP wrapper's parameter-group helpers (hl_model.py:339-394): every
    LoRA target name resolves to a Linear of the module tree, and the grad
    switches return the number of parameters they set."""
    model = Z.Z_Transformer(Z.ZImageTransformer2DModel(**Z.PRESETS["zimage-tiny"]), num_metadata=2, use_cond=True)
    mods = dict(model.named_modules())
    names = model.get_noise_lora_branch() + model.get_context_lora_branch() + model.get_main_lora_branch()
    assert len(names) == len(set(names)) > 10
    for n in names:
        assert hasattr(mods[n], "weight"), n
    n_meta = sum(p.numel() for p in model.meta_embeddings.parameters())
    assert model.switch_meta_embedding_grad(False) == n_meta
    assert not any(p.requires_grad for p in model.meta_embeddings.parameters())
    n_cond = sum(p.numel() for n, p in model.named_parameters() if n.startswith(("cond_embedder_", "cond_refiner_")))
    assert model.switch_cond_branch_grad(False) == n_cond > 0
    assert model.switch_cond_branch_grad(True) == n_cond


def test_rope_table_embedder_swap_keeps_predictions():
    """replace_ropeembedder_with_sverope swaps the Z-Image model's rotary
    embedder for the table-lookup one: bitwise the same predictions."""
    torch.manual_seed(0)
    pre = Z.PRESETS["zimage-tiny"]
    model = Z.ZImageTransformer2DModel(**pre)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0, 0.05)
    x = [torch.randn(16, 1, 18, 18)]
    caps = [torch.randn(20, pre["cap_feat_dim"])]
    t = torch.rand(1)
    with torch.no_grad():
        a = model(x, t, caps)["sample"][0]
        Z.replace_ropeembedder_with_sverope(model)
        assert isinstance(model.rope_embedder, Z.RopeTableEmbedder)
        b = model(x, t, caps)["sample"][0]
    torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_zimage_gradient_checkpointing_gives_the_same_gradients():
    """gradient_checkpointing_enable() (the reference's ModelMixin switch, a
    no-op there) recomputes each block in the backward here: the same loss and
    bitwise the same gradients for the base model and the SP wrapper, with
    padded runs and a condition branch."""
    pre = Z.PRESETS["zimage-tiny"]

    def run(ckpt, wrapper):
        torch.manual_seed(0)
        base = Z.ZImageTransformer2DModel(**pre)
        model = Z.Z_Transformer(base, num_metadata=2, use_cond=True) if wrapper else base
        with torch.no_grad():
            for p in model.parameters():
                p.normal_(0, 0.05)
        model = model.bfloat16()
        if ckpt:
            model.gradient_checkpointing_enable()
        g = torch.Generator().manual_seed(1)
        x = [torch.randn(16, 1, 18, 18, generator=g).bfloat16() for _ in range(2)]
        caps = [torch.randn(20, pre["cap_feat_dim"], generator=g).bfloat16() for _ in range(2)]
        t = torch.rand(2, generator=g)
        if wrapper:
            meta = torch.rand(2, 2, generator=g).bfloat16()
            cond = [torch.randn(2, 192, 18, 18, generator=g).bfloat16()]
            pred, _, _ = model.forward_local(x, t, caps, metadata=meta, cond_list=cond, sp=SPContext())
            loss = pred.float().pow(2).mean()
        else:
            loss = sum(o.float().pow(2).mean() for o in model(x, t, caps)["sample"])
        loss.backward()
        return loss.detach(), [p.grad.clone() if p.grad is not None else None for p in model.parameters()]

    for wrapper in (False, True):
        (l0, g0), (l1, g1) = run(False, wrapper), run(True, wrapper)
        torch.testing.assert_close(l1, l0, rtol=0, atol=0)
        for a, b in zip(g0, g1):
            assert (a is None) == (b is None)
            if a is not None:
                torch.testing.assert_close(b, a, rtol=0, atol=0)
