"""tcgen05 flash attention (forward, backward, chunked ring order) vs fp32 PyTorch."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import harp_b200

    assert harp_b200.load_native(build_if_needed=True)


def _ref_attn(q, k, v, scale):
    # q: [B, Sq, H, D] fp32
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    p = torch.softmax(s, -1)
    o = torch.einsum("bhqk,bkhd->bqhd", p, v)
    lse = torch.logsumexp(s, -1)  # [B, H, Sq]
    return o, lse


def _make(B, Sq, Skv, H, Dh, fused=True):
    g = torch.Generator(device="cuda").manual_seed(1)
    if fused and Sq == Skv:
        qkv = torch.randn(B * Sq, 3 * H * Dh, device="cuda", generator=g).to(torch.bfloat16)
        return qkv[:, : H * Dh], qkv[:, H * Dh : 2 * H * Dh], qkv[:, 2 * H * Dh :]
    q = torch.randn(B * Sq, H * Dh, device="cuda", generator=g).to(torch.bfloat16)
    kv = torch.randn(B * Skv, 2 * H * Dh, device="cuda", generator=g).to(torch.bfloat16)
    return q, kv[:, : H * Dh], kv[:, H * Dh :]


def _ld(S):
    return (S + 127) // 128 * 128


def _fwd(q, k, v, B, Sq, Skv, H, Dh, ready=None, chunk_len=0, start_tile=0, epoch=0):
    o = torch.empty(B * Sq, H * Dh, device="cuda", dtype=torch.bfloat16)
    lse = torch.full((B * H * _ld(Sq),), float("inf"), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    scale = 1.0 / math.sqrt(Dh)
    torch.ops.harp.attn_fwd(q, k, v, B, Sq, Skv, H, Dh, scale, o, lse, ready, chunk_len, start_tile, epoch, 5.0, err)
    torch.cuda.synchronize()
    assert err.cpu()[0].item() == 0, err.cpu().tolist()
    return o, lse


@pytest.mark.parametrize("Dh", [64, 72, 128])
@pytest.mark.parametrize("B,Sq,Skv,H", [(1, 128, 128, 1), (2, 300, 300, 3), (1, 200, 520, 2), (2, 544, 544, 2)])
def test_attn_fwd(B, Sq, Skv, H, Dh):
    q, k, v = _make(B, Sq, Skv, H, Dh)
    o, lse = _fwd(q, k, v, B, Sq, Skv, H, Dh)
    scale = 1.0 / math.sqrt(Dh)
    ro, rlse = _ref_attn(q.float().view(B, Sq, H, Dh), k.float().view(B, Skv, H, Dh), v.float().view(B, Skv, H, Dh), scale)
    err = (o.float().view(B, Sq, H, Dh) - ro).abs().max().item()
    assert err < 2e-2, err
    lerr = (lse.view(B, H, -1)[:, :, :Sq] - rlse).abs().max().item()
    assert lerr < 2e-2, lerr


def test_attn_fwd_chunked_ring_order():
    """Gathered K/V made of 4 chunks with readiness flags; visiting order starts mid-sequence."""
    B, Sq, H, Dh, P = 2, 160, 2, 72, 4
    Skv = Sq * P
    q, k, v = _make(B, Sq, Skv, H, Dh, fused=False)
    ready = torch.full((P,), 3, dtype=torch.int32, device="cuda")
    o, lse = _fwd(q, k, v, B, Sq, Skv, H, Dh, ready=ready, chunk_len=Sq, start_tile=(2 * Sq) // 128, epoch=3)
    o2, lse2 = _fwd(q, k, v, B, Sq, Skv, H, Dh)
    assert (o.float() - o2.float()).abs().max() < 1e-2
    assert (lse.view(B, H, -1)[:, :, :Sq] - lse2.view(B, H, -1)[:, :, :Sq]).abs().max() < 1e-3


@pytest.mark.parametrize("Dh", [72, 128])
def test_attn_fwd_queries_by_chunk_rotated(Dh):
    """Queries and keys both arrive by chunk (the fused Ulysses exchange): the
    grid visits query pairs starting at q_rot and waits for each query chunk's
    flag too; the result equals the plain forward."""
    B, H, P, C = 2, 3, 4, 272
    S = P * C
    q, k, v = _make(B, S, S, H, Dh)
    ready = torch.full((P,), 5, dtype=torch.int32, device="cuda")
    o = torch.empty(B * S, H * Dh, device="cuda", dtype=torch.bfloat16)
    lse = torch.full((B * H * _ld(S),), float("inf"), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.ops.harp.attn_fwd(q, k, v, B, S, S, H, Dh, 1.0 / math.sqrt(Dh), o, lse, ready, C, (2 * C) // 128, 5, 5.0,
                            err, (2 * C) // 256, True)
    torch.cuda.synchronize()
    assert err.cpu()[0].item() == 0, err.cpu().tolist()
    o2, lse2 = _fwd(q, k, v, B, S, S, H, Dh)
    assert (o.float() - o2.float()).abs().max() < 1e-2
    assert (lse.view(B, H, -1)[:, :, :S] - lse2.view(B, H, -1)[:, :, :S]).abs().max() < 1e-3


def test_attn_fwd_ready_timeout_reports_error():
    """A chunk flag that never arrives ends the kernel with an error word, not a hang."""
    B, Sq, H, Dh, P = 1, 128, 1, 64, 2
    q, k, v = _make(B, Sq, Sq * P, H, Dh, fused=False)
    ready = torch.tensor([1, 0], dtype=torch.int32, device="cuda")  # chunk 1 never ready
    o = torch.empty(B * Sq, H * Dh, device="cuda", dtype=torch.bfloat16)
    lse = torch.full((B * H * _ld(Sq),), float("inf"), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.ops.harp.attn_fwd(q, k, v, B, Sq, Sq * P, H, Dh, 0.125, o, lse, ready, Sq, 0, 1, 0.5, err)
    torch.cuda.synchronize()
    e = err.cpu().tolist()
    assert e[0] == 2 and e[1] == 20, e  # kErrPeerTimeout at the TMA warp's readiness wait
    # the context is still usable
    o2, _ = _fwd(q, k, v, B, Sq, Sq, H, Dh)
    assert torch.isfinite(o2.float()).all()


@pytest.mark.parametrize("Dh", [64, 72, 128])
@pytest.mark.parametrize("B,Sq,Skv,H", [(1, 128, 128, 1), (2, 300, 300, 2), (1, 200, 330, 2), (1, 1100, 700, 2)])
def test_attn_bwd(B, Sq, Skv, H, Dh):
    q, k, v = _make(B, Sq, Skv, H, Dh)
    o, lse = _fwd(q, k, v, B, Sq, Skv, H, Dh)
    scale = 1.0 / math.sqrt(Dh)
    do = torch.randn(B * Sq, H * Dh, device="cuda").to(torch.bfloat16)
    delta = torch.zeros(B * H * _ld(Sq), device="cuda")
    torch.ops.harp.rowdot(do, o, H, Dh, Sq, delta)
    dq_acc = torch.zeros(B * H * Sq * Dh, device="cuda")  # [B, H, Sq, Dh]
    dk = torch.empty(B * Skv, H * Dh, device="cuda", dtype=torch.bfloat16)
    dv = torch.empty_like(dk)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.ops.harp.attn_bwd(q, k, v, do, lse, delta, B, Sq, Skv, H, Dh, scale, dq_acc, dk, dv, err)
    dq = torch.empty(B * Sq, H * Dh, device="cuda", dtype=torch.bfloat16)
    torch.ops.harp.dq_finalize(dq_acc, H, Dh, scale, dq, Sq)
    torch.cuda.synchronize()
    assert err.cpu()[0].item() == 0, err.cpu().tolist()
    qr = q.float().view(B, Sq, H, Dh).requires_grad_()
    kr = k.float().view(B, Skv, H, Dh).requires_grad_()
    vr = v.float().view(B, Skv, H, Dh).requires_grad_()
    ro, _ = _ref_attn(qr, kr, vr, scale)
    ro.backward(do.float().view(B, Sq, H, Dh))
    for name, got, ref in [("dq", dq, qr.grad), ("dk", dk, kr.grad), ("dv", dv, vr.grad)]:
        g = got.float().view_as(ref)
        e = (g - ref).abs().max().item()
        tol = 3e-2 * max(1.0, ref.abs().max().item())
        assert e < tol, (name, e, tol)


def test_exp2_poly_error_bound():
    """The FMA-pipe 2^x of the softmax against fp32 exp2: relative error below
    1e-4 over the range the softmax produces (clamped at -125)."""
    x = torch.cat([torch.linspace(-125.0, 8.0, 1_000_001, device="cuda"),
                   torch.rand(1_000_000, device="cuda") * -30.0])
    y = torch.ops.harp.exp2_poly(x)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref) / ref).abs().max().item()
    assert rel < 1e-4, rel
    z = torch.ops.harp.exp2_poly(torch.tensor([-float("inf"), -1000.0, 0.0], device="cuda"))
    assert z[0].item() < 1e-37 and z[1].item() < 1e-37 and z[2].item() == pytest.approx(1.0, rel=1e-4)


@pytest.mark.parametrize("npoly", ["6", "16"])
def test_attn_fwd_poly_exp(npoly):
    """Forward attention with part (or all) of the softmax exponentials on the
    polynomial: same result as the fp32 reference within bf16 tolerance."""
    import subprocess
    import sys

    code = (
        "import torch, harp_b200\n"
        "from harp_b200.ops import functional as Fn\n"
        "harp_b200.load_native(build_if_needed=False)\n"
        "torch.manual_seed(0)\n"
        "B, S, H, Dh = 2, 700, 3, 72\n"
        "q, k, v = (torch.randn(B*S, H*Dh, device='cuda').bfloat16() for _ in range(3))\n"
        "o, lse = Fn.attn_fwd(q, k, v, B, S, S, H, Dh)\n"
        "qf, kf, vf = (t.float().view(B, S, H, Dh).transpose(1, 2) for t in (q, k, v))\n"
        "ref = torch.softmax(qf @ kf.transpose(-1, -2) / Dh**0.5, -1) @ vf\n"
        "err = (o.float().view(B, S, H, Dh).transpose(1, 2) - ref).abs().max().item()\n"
        "assert err < 2e-2, err\n"
        "print('ok', err)\n"
    )
    import os

    env = dict(os.environ, HARP_ATTN_POLY=npoly)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("env", [{"HARP_ATTN_BWD_Q64": "all"}, {"HARP_ATTN_FWD": "split"},
                                 {"HARP_ATTN_BWD_PAIR": "1"}])
def test_attention_alternative_schedules(env):
    """The schedules chosen by environment variables (read once per process):
    the 64-query-tile backward for head dims 64-80, the two-warps-per-row
    forward, and the backward kernels in CTA pairs that combine dQ partials
    through distributed shared memory, run through the same checks in a child
    process."""
    import os
    import subprocess
    import sys

    if os.environ.get("HARP_ATTN_CHILD"):
        pytest.skip("already inside the child run")
    child_env = dict(os.environ, HARP_ATTN_CHILD="1", **env)
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-x", "-q", "-k", "test_attn_bwd or test_attn_fwd"],
                       env=child_env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
