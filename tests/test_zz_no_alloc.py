"""The allocation-free RMSNorm backward entry point (C symbol
``harp_rmsnorm_backward_noalloc``) against the library's allocating one
(``async_op::rmsnorm_backward_out``).

It serves callers that cannot call cudaMalloc while they run (plugins of
engines that plan all device memory ahead, processes whose memory is fully
reserved by a pool); its scratch is a fixed static device array, so this
test calls it through the exported symbol twice in a row, with different
shapes, to show that the shared scratch carries nothing over between calls.
The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import harp_b200
    from harp_b200 import _native

    assert harp_b200.load_native(build_if_needed=True)
    lib = ctypes.CDLL(_native.so_path())
    fn = lib.harp_rmsnorm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_void_p]
    return fn


def _case(fn, rows, dim, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.rand(dim, device="cuda", generator=g) + 0.5).to(torch.bfloat16)
    y = torch.empty_like(x)
    rms = torch.empty(rows, device="cuda")
    torch.ops.async_op.rmsnorm_forward_out(x, w, y, rms, 1e-6)
    # existing entry point (allocates its scratch through PyTorch)
    gi_ref = torch.empty_like(x)
    gw_ref = torch.empty_like(w)
    torch.ops.async_op.rmsnorm_backward_out(x, dy, w, rms, gi_ref, gw_ref)
    # allocation-free entry point, through its exported C symbol
    gi = torch.full_like(x, float("nan"))
    gw = torch.full_like(w, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(x.data_ptr(), dy.data_ptr(), w.data_ptr(), rms.data_ptr(), gi.data_ptr(), gw.data_ptr(), rows, dim,
            ctypes.c_void_p(stream))
    torch.cuda.synchronize()
    assert rc == 0, rc
    assert (gi.float() - gi_ref.float()).abs().max().item() < 0.05
    assert torch.allclose(gw.float(), gw_ref.float(), atol=0.5, rtol=2e-2)


def test_noalloc_rmsnorm_backward_matches_allocating_entry():
    fn = _lib()
    _case(fn, rows=3000, dim=1152, seed=1)  # first call also sets up the scratch address
    _case(fn, rows=517, dim=384, seed=2)  # second call: different shape over the same scratch


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
