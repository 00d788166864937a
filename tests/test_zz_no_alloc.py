"""The allocation-free RMSNorm backward entry point (C symbol
``harp_rmsnorm_backward_noalloc``, declared in ``harp_b200/csrc/harp_noalloc.h``).

It serves callers that cannot call cudaMalloc while they run: plugins of engines
that plan all device memory ahead, processes whose memory a pool has fully
reserved, loops that cannot afford an allocation's device synchronisation.  Its
only scratch is a fixed static device array shared by every call, so this test
calls it through the exported symbol several times in a row, each call checked
against both the library's allocating entry (``async_op::rmsnorm_backward_out``)
and an fp32 PyTorch autograd RMSNorm backward of the same inputs.  The calls run
smaller footprint first, then one that fills far more of the scratch, then an
empty batch, so that nothing can carry over from one call to the next unseen.
The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _lib():
    import harp_b200
    from harp_b200 import _native

    assert harp_b200.load_native(build_if_needed=True)
    lib = ctypes.CDLL(_native.so_path())
    fn = lib.harp_rmsnorm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_void_p]
    return fn


def _fp32_reference(x, dy, w):
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * wf
    y.backward(dy.float())
    return xf.grad, wf.grad


def _case(fn, rows, dim, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.rand(dim, device="cuda", generator=g) + 0.5).to(torch.bfloat16)
    y = torch.empty_like(x)
    rms = torch.empty(rows, device="cuda")
    if rows:
        torch.ops.async_op.rmsnorm_forward_out(x, w, y, rms, EPS)
    # existing entry point (allocates its scratch through PyTorch)
    gi_ref = torch.empty_like(x)
    gw_ref = torch.empty_like(w)
    if rows:
        torch.ops.async_op.rmsnorm_backward_out(x, dy, w, rms, gi_ref, gw_ref)
    # allocation-free entry point, through its exported C symbol
    gi = torch.full_like(x, float("nan"))
    gw = torch.full_like(w, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(x.data_ptr(), dy.data_ptr(), w.data_ptr(), rms.data_ptr(), gi.data_ptr(), gw.data_ptr(), rows, dim,
            ctypes.c_void_p(stream))
    torch.cuda.synchronize()
    assert rc == 0, rc
    if rows == 0:
        assert torch.equal(gw.float(), torch.zeros(dim, device="cuda"))
        return
    # against the allocating entry point
    torch.testing.assert_close(gi.float(), gi_ref.float(), atol=0.05, rtol=2e-2)
    torch.testing.assert_close(gw.float(), gw_ref.float(), atol=0.5, rtol=2e-2)
    # against fp32 autograd: bf16 rounding of the outputs (2^-8 relative)
    dxr, dwr = _fp32_reference(x, dy, w)
    torch.testing.assert_close(gi.float(), dxr, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(gw.float(), dwr, atol=5e-2, rtol=1e-2)


def test_noalloc_rmsnorm_backward_matches_allocating_entry_and_fp32():
    fn = _lib()
    _case(fn, rows=517, dim=384, seed=2)  # first call also sets up the scratch address
    _case(fn, rows=3000, dim=1152, seed=1)
    # 40000 x 1024 needs more rows per block than 32 (the scratch holds 1024
    # partial rows of this width): the path with up to 4096 rows per block and
    # a larger shared-memory row-statistics buffer, filling the whole scratch
    _case(fn, rows=40000, dim=1024, seed=3)
    _case(fn, rows=0, dim=1024, seed=4)  # empty batch: grad_weight is zero
    _case(fn, rows=5000, dim=8, seed=5)  # narrow rows: block count bounded by the row target


def test_noalloc_rejects_bad_sizes():
    fn = _lib()
    x = torch.zeros(4, 16, device="cuda", dtype=torch.bfloat16)
    rms = torch.ones(4, device="cuda")
    w = torch.ones(16, device="cuda", dtype=torch.bfloat16)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # dim not a multiple of 8
    assert fn(x.data_ptr(), x.data_ptr(), w.data_ptr(), rms.data_ptr(), x.data_ptr(), w.data_ptr(), 4, 12, s) == -1
    # more rows than the static scratch can hold for this dim: rejected before any launch
    assert fn(x.data_ptr(), x.data_ptr(), w.data_ptr(), rms.data_ptr(), x.data_ptr(), w.data_ptr(),
              1 << 40, 1 << 19, s) == -2
