"""Run-to-run determinism of the kernels that reduce in a fixed order: the same
inputs give bit-identical outputs twice.  Covers the GEMM (both CTA schedules),
RMSNorm + modulation forward/backward with their column partial sums, the gated
residual backward, SwiGLU, and attention forward and the dK/dV of its backward
(accumulated in tensor memory in query-tile order).  The attention backward's
dQ is left out on purpose: its per-key-tile partials are reduce-added in L2 in
no fixed order."""
import pytest
import torch

import harp_b200
from harp_b200.ops import functional as Fn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert harp_b200.load_native(build_if_needed=True), "CUDA library must load on a GPU box"


def _twice(fn):
    torch.manual_seed(0)
    a = fn()
    b = fn()
    torch.cuda.synchronize()
    return a, b


def _same(a, b):
    for x, y in zip(a, b):
        if x is None:
            assert y is None
            continue
        assert torch.equal(x, y), (x.float() - y.float()).abs().max().item()


@pytest.mark.parametrize("pair", [0, 1])
def test_linear_forward_backward_bit_identical(pair):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2176, 1152, device="cuda", generator=g).bfloat16()
    w = torch.randn(4608, 1152, device="cuda", generator=g).bfloat16()
    b = torch.randn(4608, device="cuda", generator=g).bfloat16()
    dy = torch.randn(2176, 4608, device="cuda", generator=g).bfloat16()
    prev = torch.ops.harp.gemm_pair_mode(pair)
    try:
        a, c = _twice(lambda: (Fn.linear_fwd(x, w, b),) + Fn.linear_bwd(dy, x, w, True))
    finally:
        torch.ops.harp.gemm_pair_mode(prev)
    _same(a, c)


def test_rmsnorm_gate_swiglu_bit_identical():
    g = torch.Generator(device="cuda").manual_seed(2)
    Bn, S, D, F_ = 4, 544, 1152, 4608
    R = Bn * S
    x = torch.randn(R, D, device="cuda", generator=g).bfloat16()
    w = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    mod = (torch.randn(Bn, 2 * D, device="cuda", generator=g) * 0.5).bfloat16()
    dy = torch.randn(R, D, device="cuda", generator=g).bfloat16()
    a = torch.randn(R, D, device="cuda", generator=g).bfloat16()
    gate = torch.randn(Bn, D, device="cuda", generator=g).bfloat16()
    gu = torch.randn(R, 2 * F_, device="cuda", generator=g).bfloat16()
    dh = torch.randn(R, F_, device="cuda", generator=g).bfloat16()

    def run():
        y, rstd = Fn.rmsnorm_mod_fwd(x, w, mod[:, :D], mod[:, D:], S, 1e-6)
        dx, dw, ds, dsh = Fn.rmsnorm_mod_bwd(x, rstd, dy, w, mod[:, :D], S, want_dw=True, want_mod=True)
        da, dgate, dbias = Fn.gate_bwd(dy, a, gate, S)
        h = Fn.swiglu_fwd(gu, F_)
        dgu = Fn.swiglu_bwd(dh, gu)
        return y, rstd, dx, dw, ds, dsh, da, dgate, dbias, h, dgu

    first, second = _twice(run)
    _same(first, second)


@pytest.mark.parametrize("Dh,H", [(72, 4), (128, 3)])
def test_attention_forward_and_dkdv_bit_identical(Dh, H):
    g = torch.Generator(device="cuda").manual_seed(3)
    B, S = 2, 1088
    q, k, v, do = (torch.randn(B * S, H * Dh, device="cuda", generator=g).bfloat16() for _ in range(4))

    def run():
        o, lse = Fn.attn_fwd(q, k, v, B, S, S, H, Dh)
        _, dk, dv = Fn.attn_bwd(q, k, v, o, do, lse, B, S, S, H, Dh)
        return o, lse, dk, dv

    first, second = _twice(run)
    _same(first, second)
