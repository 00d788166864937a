"""Every model family through the CUDA kernels (tcgen05 GEMM, flash attention,
fused norms) against the same model run through the fp32 CPU restatements."""
import copy

import pytest
import torch

from harp_b200.models import dit as D
from harp_b200.models import mmdit as M
from harp_b200.models import zimage as Z
from harp_b200.parallel.sequence import SPContext

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _compare(build, loss_fn, inputs, tol=3e-2):
    torch.manual_seed(0)
    cpu = build()
    with torch.no_grad():
        for p in cpu.parameters():
            p.normal_(0, 0.05)
    cpu = cpu.to(torch.bfloat16)
    gpu = copy.deepcopy(cpu).cuda()
    lc = loss_fn(cpu, *inputs)
    lc.backward()
    lg = loss_fn(gpu, *[x.cuda() if isinstance(x, torch.Tensor) else [y.cuda() for y in x] for x in inputs])
    lg.backward()
    torch.cuda.synchronize()
    assert abs(lg.item() - lc.item()) <= tol * abs(lc.item()), (lg.item(), lc.item())
    worst = max(((_rel(pg.grad, pc.grad), n) for (n, pc), pg in zip(cpu.named_parameters(), gpu.parameters())
                 if pc.grad is not None and pc.grad.float().norm() > 0), default=(0.0, ""))
    assert worst[0] < 8e-2, worst


def _common(C=16, L=16, T=32, Dt=128, B=2):
    g = torch.Generator().manual_seed(1)
    lat = torch.randn(B, C, L, L, generator=g).bfloat16()
    return lat, torch.randn(B, C, L, L, generator=g).bfloat16(), torch.randn(B, T, Dt, generator=g).bfloat16(), \
        torch.rand(B, generator=g)


def test_dit_small_cuda_matches_cpu():
    cfg = D.PRESETS["small"]
    lat, noise, text, sig = _common(C=cfg.in_channels, Dt=cfg.text_dim)
    _compare(lambda: D.DiT(cfg), lambda m, a, b, c, d: D.flow_matching_loss_local(m, a, b, c, d, SPContext()),
             (lat, noise, text, sig))


@pytest.mark.parametrize("name", ["mmdit-tiny", "flux-tiny"])
def test_mmdit_family_cuda_matches_cpu(name):
    cfg = M.PRESETS[name]
    lat, noise, text, sig = _common(Dt=cfg.text_dim)
    _compare(lambda: M.MMDiT(cfg), lambda m, a, b, c, d: M.mmdit_loss_local(m, a, b, c, d, SPContext()),
             (lat, noise, text, sig))


def test_zimage_cuda_matches_cpu():
    pre = Z.PRESETS["zimage-tiny"]
    lat, noise, text, sig = _common(Dt=pre["cap_feat_dim"])
    g = torch.Generator().manual_seed(2)
    meta = torch.rand(2, 4, generator=g).bfloat16()
    cond = [torch.randn(2, 192, 16, 16, generator=g).bfloat16()]
    _compare(lambda: Z.Z_Transformer(Z.ZImageTransformer2DModel(**pre), num_metadata=4, use_cond=True),
             lambda m, a, b, c, d, e, f: Z.zimage_loss_local(m, a, b, c, d, SPContext(), metadata=e, cond=f),
             (lat, noise, text, sig, meta, cond))
