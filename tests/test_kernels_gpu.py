"""Numerics of the sm_100a kernels against plain PyTorch fp32 references.

Each CUDA kernel is compared with an fp32 restatement of the same op; shapes
include tails (M, N, K not multiples of the tile) to exercise the TMA
out-of-bounds fill and the epilogue masks.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import harp_b200

    assert harp_b200.load_native(build_if_needed=True), "CUDA library must load on a GPU box"
    torch.manual_seed(0)


def _err():
    return torch.zeros(4, dtype=torch.int32, device="cuda")


def _check_err(err):
    e = err.cpu().tolist()
    assert e[0] == 0, f"device error word {e}"


def _gemm(A, a_mn, B, b_mn, M, N, K, epi=0, bias=None, alpha=1.0, residual=None, gate=None, rpb=0, C=None,
          force_simt=False):
    out_dtype = torch.float32 if epi in (1, 3) else torch.bfloat16
    if C is None:
        C = torch.zeros(M, N, dtype=out_dtype, device="cuda")
    err = _err()
    torch.ops.harp.gemm(A, a_mn, B, b_mn, C, M, N, K, bias, epi, alpha, residual, gate, rpb, err, force_simt)
    torch.cuda.synchronize()
    _check_err(err)
    return C


def _ref(A, a_mn, B, b_mn):
    a = A.float().t() if a_mn else A.float()
    b = B.float() if b_mn else B.float().t()
    return a @ b


SHAPES = [(128, 256, 64), (256, 512, 256), (300, 200, 136), (1000, 1152, 1152), (64, 3456, 1152), (17, 40, 24),
          (2176, 4608, 1152)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_majors(M, N, K, a_mn, b_mn):
    A = (torch.randn(K, M) if a_mn else torch.randn(M, K)).to(torch.bfloat16).cuda()
    B = (torch.randn(K, N) if b_mn else torch.randn(N, K)).to(torch.bfloat16).cuda()
    C = _gemm(A, a_mn, B, b_mn, M, N, K)
    ref = _ref(A, a_mn, B, b_mn)
    tol = 2e-2 * math.sqrt(K) + 1e-2
    assert (C.float() - ref).abs().max().item() < tol, (C.float() - ref).abs().max().item()


PAIR_SHAPES = [(512, 256, 64), (600, 300, 200), (1000, 1152, 1152), (2176, 4608, 1152), (4352, 1152, 4608),
               (768, 640, 72)]


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_cta_pair_matches_single(M, N, K, a_mn, b_mn):
    """The CTA-pair (cta_group::2) kernel and the single-CTA kernel against fp32."""
    A = (torch.randn(K, M) if a_mn else torch.randn(M, K)).to(torch.bfloat16).cuda()
    B = (torch.randn(K, N) if b_mn else torch.randn(N, K)).to(torch.bfloat16).cuda()
    ref = _ref(A, a_mn, B, b_mn)
    tol = 2e-2 * math.sqrt(K) + 1e-2
    prev = torch.ops.harp.gemm_pair_mode(1)
    try:
        c_pair = _gemm(A, a_mn, B, b_mn, M, N, K, epi=1)
        torch.ops.harp.gemm_pair_mode(0)
        c_one = _gemm(A, a_mn, B, b_mn, M, N, K, epi=1)
    finally:
        torch.ops.harp.gemm_pair_mode(prev)
    assert (c_pair - ref).abs().max().item() < tol
    assert (c_one - ref).abs().max().item() < tol
    # same products summed in the same k order: fp32 results agree closely
    assert (c_pair - c_one).abs().max().item() < 1e-3 * math.sqrt(K)


@pytest.mark.parametrize("pair", [0, 1])
def test_gemm_epilogues_modes(pair):
    prev = torch.ops.harp.gemm_pair_mode(pair)
    try:
        test_gemm_epilogues()
    finally:
        torch.ops.harp.gemm_pair_mode(prev)


def test_gemm_epilogues():
    M, N, K, B_ = 512, 384, 192, 4
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    W = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, device="cuda").to(torch.bfloat16)
    ref = A.float() @ W.float().t() + bias.float()
    c = _gemm(A, False, W, False, M, N, K, epi=0, bias=bias)
    assert (c.float() - ref).abs().max() < 0.5
    c32 = _gemm(A, False, W, False, M, N, K, epi=1, bias=bias)
    assert (c32 - ref).abs().max() < 0.05
    acc = torch.randn(M, N, device="cuda")
    acc0 = acc.clone()
    _gemm(A, False, W, False, M, N, K, epi=3, bias=bias, C=acc)
    assert (acc - (acc0 + ref)).abs().max() < 0.05
    res = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    gate = torch.randn(B_, N, device="cuda").to(torch.bfloat16)
    out = _gemm(A, False, W, False, M, N, K, epi=4, bias=bias, residual=res, gate=gate, rpb=M // B_)
    gref = res.float() + gate.float().repeat_interleave(M // B_, 0) * ref
    assert (out.float() - gref).abs().max() < 1.0


def test_gemm_simt_fallback_matches():
    M, N, K = 100, 72, 40
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    W = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    c1 = _gemm(A, False, W, False, M, N, K, force_simt=True)
    ref = A.float() @ W.float().t()
    assert (c1.float() - ref).abs().max() < 0.2


def _rms_ref(x, w, scale, shift, rpb, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if w is not None:
        y = y * w.float()
    if scale is not None:
        y = y * (1 + scale.float().repeat_interleave(rpb, 0))
    if shift is not None:
        y = y + shift.float().repeat_interleave(rpb, 0)
    return y


@pytest.mark.parametrize("D,use_dres", [(1152, False), (1152, True), (2304, True), (1000, True)])
@pytest.mark.parametrize("use_w,use_mod", [(True, False), (False, True), (True, True)])
def test_rmsnorm_mod_fwd_bwd(use_w, use_mod, D, use_dres):
    """D=1152 and D=2304 run the register-resident forward and the row-parallel
    backward, D=1000 the column-parallel ones."""
    Bn, S, eps = 3, 96, 1e-6
    R = Bn * S
    x = torch.randn(R, D, device="cuda").to(torch.bfloat16)
    w = (torch.rand(D, device="cuda") + 0.5).to(torch.bfloat16) if use_w else None
    mod = torch.randn(Bn, 2 * D, device="cuda").to(torch.bfloat16) * 0.5 if use_mod else None
    scale = mod[:, :D] if use_mod else None
    shift = mod[:, D:] if use_mod else None
    y = torch.empty_like(x)
    rstd = torch.empty(R, device="cuda")
    torch.ops.harp.rmsnorm_mod_fwd(x, w, scale, shift, S, eps, y, rstd, False)
    ref = _rms_ref(x, w, scale, shift, S, eps)
    assert (y.float() - ref).abs().max() < 0.08
    # backward
    dy = torch.randn(R, D, device="cuda").to(torch.bfloat16)
    rpb = torch.ops.harp.rows_per_block(S)
    nblk = R // rpb
    pw = torch.empty(nblk, D, device="cuda") if use_w else None
    ps = torch.empty(nblk, D, device="cuda") if use_mod else None
    pb = torch.empty(nblk, D, device="cuda") if use_mod else None
    dx = torch.empty_like(x)
    dres = torch.randn(R, D, device="cuda").to(torch.bfloat16) if use_dres else None
    torch.ops.harp.rmsnorm_mod_bwd(x, rstd, dy, w, scale, S, dres, dx, pw, ps, pb, rpb)
    if use_dres:
        dx = (dx.float() - dres.float()).to(torch.bfloat16)
    xr = x.float().requires_grad_()
    wr = w.float().requires_grad_() if use_w else None
    scr = scale.float().requires_grad_() if use_mod else None
    shr = shift.float().requires_grad_() if use_mod else None
    yr = _rms_ref(xr, wr, scr, shr, S, eps)
    yr.backward(dy.float())
    assert (dx.float() - xr.grad).abs().max() < 0.1
    if use_w:
        gw = torch.empty(1, D, device="cuda")
        torch.ops.harp.reduce_partials(pw, nblk, gw, False)
        assert torch.allclose(gw[0], wr.grad, atol=0.5, rtol=2e-2)
    if use_mod:
        gs = torch.empty(Bn, D, device="cuda")
        gb = torch.empty(Bn, D, device="cuda")
        torch.ops.harp.reduce_partials(ps, S // rpb, gs, False)
        torch.ops.harp.reduce_partials(pb, S // rpb, gb, False)
        assert torch.allclose(gs, scr.grad, atol=0.5, rtol=2e-2)
        assert torch.allclose(gb, shr.grad, atol=0.5, rtol=2e-2)


def _rope_ref(x, cos, sin):
    x0, x1 = x[..., 0::2], x[..., 1::2]
    o0 = x0 * cos - x1 * sin
    o1 = x0 * sin + x1 * cos
    return torch.stack([o0, o1], -1).flatten(-2)


@pytest.mark.parametrize("Dh", [64, 72, 128])
def test_qknorm_rope(Dh):
    R, H, eps = 200, 4, 1e-5
    qkv = torch.randn(R, 3 * H * Dh, device="cuda").to(torch.bfloat16)
    wq = (torch.rand(Dh, device="cuda") + 0.5).to(torch.bfloat16)
    wk = (torch.rand(Dh, device="cuda") + 0.5).to(torch.bfloat16)
    ang = torch.rand(R, Dh // 2, device="cuda") * 6.0
    freqs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    qo = torch.empty(R, H * Dh, device="cuda", dtype=torch.bfloat16)
    ko = torch.empty_like(qo)
    rq = torch.empty(R * H, device="cuda")
    rk = torch.empty(R * H, device="cuda")
    torch.ops.harp.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, R, eps, True, qo, ko, rq, rk)

    def ref(xpart, w):
        xr = xpart.view(R, H, Dh)
        n = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps) * w
        return _rope_ref(n, ang.cos()[:, None], ang.sin()[:, None]).reshape(R, H * Dh)

    q_in = qkv[:, : H * Dh].float().requires_grad_()
    k_in = qkv[:, H * Dh : 2 * H * Dh].float().requires_grad_()
    wqr = wq.float().requires_grad_()
    wkr = wk.float().requires_grad_()
    qr, kr = ref(q_in, wqr), ref(k_in, wkr)
    assert (qo.float() - qr).abs().max() < 0.05
    assert (ko.float() - kr).abs().max() < 0.05
    dq = torch.randn_like(qo)
    dk = torch.randn_like(ko)
    dqkv = torch.zeros_like(qkv)
    ipb = 64
    nblk = (R * H + ipb - 1) // ipb
    pwq = torch.empty(nblk, Dh, device="cuda")
    pwk = torch.empty(nblk, Dh, device="cuda")
    torch.ops.harp.qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, R, True, dqkv, pwq, pwk, ipb)
    (qr * dq.float()).sum().add((kr * dk.float()).sum()).backward()
    assert (dqkv[:, : H * Dh].float() - q_in.grad).abs().max() < 0.05
    assert (dqkv[:, H * Dh : 2 * H * Dh].float() - k_in.grad).abs().max() < 0.05
    gwq = torch.empty(1, Dh, device="cuda")
    torch.ops.harp.reduce_partials(pwq, nblk, gwq, False)
    assert torch.allclose(gwq[0], wqr.grad, atol=0.3, rtol=2e-2)


def test_swiglu_and_gate_bwd():
    R, F = 256, 512
    gu = torch.randn(R, 2 * F, device="cuda").to(torch.bfloat16)
    h = torch.empty(R, F, device="cuda", dtype=torch.bfloat16)
    torch.ops.harp.swiglu_fwd(gu, h)
    g, u = gu.float()[:, :F].requires_grad_(), gu.float()[:, F:].requires_grad_()
    hr = torch.nn.functional.silu(g) * u
    assert (h.float() - hr).abs().max() < 0.05
    dh = torch.randn_like(h)
    dgu = torch.empty_like(gu)
    torch.ops.harp.swiglu_bwd(dh, gu, dgu)
    hr.backward(dh.float())
    assert (dgu[:, :F].float() - g.grad).abs().max() < 0.05
    assert (dgu[:, F:].float() - u.grad).abs().max() < 0.05



@pytest.mark.parametrize("D", [384, 1152, 2048])
def test_gate_bwd(D):
    """Gated-residual backward: D=1152 and D=2048 take the row-parallel kernel,
    D=384 the column-parallel one."""
    Bn, S = 2, 128
    dy = torch.randn(Bn * S, D, device="cuda").to(torch.bfloat16)
    a = torch.randn(Bn * S, D, device="cuda").to(torch.bfloat16)
    gate = torch.randn(Bn, D, device="cuda").to(torch.bfloat16)
    rpb = torch.ops.harp.rows_per_block(S)
    nblk = Bn * S // rpb
    da = torch.empty_like(dy)
    pg = torch.empty(nblk, D, device="cuda")
    pb = torch.empty(nblk, D, device="cuda")
    torch.ops.harp.gate_bwd(dy, a, gate, S, da, pg, pb, rpb)
    ref_da = dy.float() * gate.float().repeat_interleave(S, 0)
    assert (da.float() - ref_da).abs().max() < 0.05
    gg = torch.empty(Bn, D, device="cuda")
    torch.ops.harp.reduce_partials(pg, S // rpb, gg, False)
    ref_g = (dy.float() * a.float()).view(Bn, S, D).sum(1)
    assert torch.allclose(gg, ref_g, atol=0.3, rtol=1e-2)
    gb = torch.empty(1, D, device="cuda")
    torch.ops.harp.reduce_partials(pb, nblk, gb, False)
    assert torch.allclose(gb[0], ref_da.sum(0), atol=0.3, rtol=1e-2)


def test_adamw_flat_matches_torch():
    n = 10007
    p0 = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    master, m, v = p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    pref = p0.clone().requires_grad_()
    opt = torch.optim.AdamW([pref], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    for step in range(1, 4):
        torch.ops.harp.adamw_flat(master, m, v, g, None, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 1.0)
        pref.grad = g.clone()
        opt.step()
    assert torch.allclose(master, pref.detach(), atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("gdtype", [torch.float32, torch.bfloat16])
def test_adamw_flat_vector_path_matches_scalar_path(gdtype):
    """n % 8 == 0 with aligned buffers takes the 16-byte vector kernel; it must
    agree with the element-wise kernel to a few ulp (same per-element math, the
    compiler may contract multiply-adds differently)."""
    n = 8 * 12531
    p0 = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda").to(gdtype)
    states = []
    for length in (n, n + 1):  # n + 1: element-wise kernel on a buffer that is not a multiple of 8
        master = torch.zeros(length, device="cuda")
        master[:n] = p0
        m, v = torch.zeros_like(master), torch.zeros_like(master)
        gg = torch.zeros(length, device="cuda", dtype=gdtype)
        gg[:n] = g
        param = torch.empty(length, device="cuda", dtype=torch.bfloat16)
        for step in range(1, 4):
            torch.ops.harp.adamw_flat(master, m, v, gg, param, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 0.5)
        states.append((master[:n].clone(), m[:n].clone(), v[:n].clone(), param[:n].clone()))
    for a, b in zip(states[0][:3], states[1][:3]):
        torch.testing.assert_close(a, b, rtol=4e-6, atol=1e-7)
    torch.testing.assert_close(states[0][3].float(), states[1][3].float(), rtol=2 ** -7, atol=0.0)
    torch.testing.assert_close(states[0][3], states[0][0].to(torch.bfloat16))


def test_philox_uniform_range_and_determinism():
    a = torch.empty(100003, device="cuda")
    b = torch.empty(100003, device="cuda")
    torch.ops.harp.philox_uniform(a, 7, 0, -2.0, 3.0)
    torch.ops.harp.philox_uniform(b, 7, 0, -2.0, 3.0)
    assert torch.equal(a, b)
    assert a.min() >= -2.0 and a.max() < 3.0
    assert abs(a.mean().item() - 0.5) < 0.05


def test_compat_linear_ops():
    x = torch.randn(4, 37, 256, device="cuda").to(torch.bfloat16)
    w = torch.randn(320, 256, device="cuda").to(torch.bfloat16)
    b = torch.randn(320, device="cuda").to(torch.bfloat16)
    out = torch.empty(4, 37, 320, device="cuda", dtype=torch.bfloat16)
    torch.ops.xhpops.kp_linear_forward(x, w, b, out)
    ref = x.float() @ w.float().t() + b.float()
    assert (out.float() - ref).abs().max() < 0.5
    g = torch.randn_like(out)
    gi = torch.empty_like(x)
    gw = torch.empty_like(w)
    gb = torch.empty_like(b)
    torch.ops.xhpops.kp_linear_backward(g, x, w, gi, gw, gb)
    torch.cuda.synchronize()
    gf = g.float().view(-1, 320)
    assert (gi.float().view(-1, 256) - gf @ w.float()).abs().max() < 0.5
    assert (gw.float() - gf.t() @ x.float().view(-1, 256)).abs().max() < 2.0
    assert (gb.float() - gf.sum(0)).abs().max() < 0.5


@pytest.mark.parametrize("Dh,strided", [(72, False), (128, False), (64, True), (48, False)])
def test_qknorm_rope_bwd_paths_match_autograd(Dh, strided):
    """The functional wrapper: vectorized kernel for head_dim 64/72/80/96/128 with
    16-byte aligned rows (strided dq/dk views of a wider buffer included), the
    warp-per-item kernel otherwise; in-place use (dq aliasing the output) too."""
    from harp_b200.ops import functional as Fn

    R, H, eps = 300, 4, 1e-6
    HD = H * Dh
    qkv = torch.randn(R, 3 * HD, device="cuda").to(torch.bfloat16)
    wq = (torch.rand(Dh, device="cuda") + 0.5).to(torch.bfloat16)
    wk = (torch.rand(Dh, device="cuda") + 0.5).to(torch.bfloat16)
    ang = torch.rand(R, Dh // 2, device="cuda") * 6.0
    freqs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    q, k, rq, rk = Fn.qknorm_rope_fwd(qkv, H, Dh, wq, wk, freqs, eps)
    if strided:
        g = torch.randn(R, 3 * HD, device="cuda").to(torch.bfloat16)
        dq, dk = g[:, :HD], g[:, HD:2 * HD]
        out = g  # in place: the gradient buffer is the output buffer
    else:
        dq, dk = torch.randn_like(q), torch.randn_like(k)
        out = torch.zeros_like(qkv)
    dq_ref, dk_ref = dq.float().clone(), dk.float().clone()
    dwq, dwk = Fn.qknorm_rope_bwd(dq, dk, qkv, rq, rk, H, Dh, wq, wk, freqs, True, out)

    def ref(xpart, w):
        xr = xpart.view(R, H, Dh)
        n = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps) * w
        return _rope_ref(n, ang.cos()[:, None], ang.sin()[:, None]).reshape(R, HD)

    q_in = qkv[:, :HD].float().requires_grad_()
    k_in = qkv[:, HD:2 * HD].float().requires_grad_()
    wqr, wkr = wq.float().requires_grad_(), wk.float().requires_grad_()
    (ref(q_in, wqr) * dq_ref).sum().add((ref(k_in, wkr) * dk_ref).sum()).backward()
    assert (out[:, :HD].float() - q_in.grad).abs().max() < 0.05
    assert (out[:, HD:2 * HD].float() - k_in.grad).abs().max() < 0.05
    torch.testing.assert_close(dwq, wqr.grad, atol=0.3, rtol=2e-2)
    torch.testing.assert_close(dwk, wkr.grad, atol=0.3, rtol=2e-2)
