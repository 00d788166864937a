"""Native two-tier allocator (csrc/alloc.cpp) through torch MemPools.  torch's
caching allocator sits on top of each pool: it asks the native allocator for
segments and hands them back on empty_cache()."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_host_tier_tensors_are_device_usable_and_cached():
    from harp_b200.managers import mem_manager as MM
    from harp_b200.runtime import alloc

    before = alloc.stats("host")
    with MM.use_hbm_allocator(False):
        x = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
    s = alloc.stats("host")
    assert s["allocations"] > before["allocations"] and s["in_use"] >= 4 << 20
    y = (x * 2).sum()  # a kernel reads the host-tier tensor in place
    assert y.item() == float((1 << 20) * ((1 << 20) - 1))
    del x


def test_native_host_cache_reuses_blocks_after_their_stream_is_done():
    import ctypes

    from harp_b200.runtime import alloc

    lib = alloc._clib()
    lib.harp_host_malloc.restype = ctypes.c_void_p
    lib.harp_host_malloc.argtypes = [ctypes.c_ssize_t, ctypes.c_int, ctypes.c_void_p]
    lib.harp_host_free.argtypes = [ctypes.c_void_p, ctypes.c_ssize_t, ctypes.c_int, ctypes.c_void_p]
    stream = torch.cuda.current_stream().cuda_stream
    s0 = alloc.stats("host")
    p = lib.harp_host_malloc(3 << 20, 0, stream)  # 4 MiB size class
    assert p
    lib.harp_host_free(p, 3 << 20, 0, stream)
    torch.cuda.synchronize()
    s1 = alloc.stats("host")
    assert s1["cached"] >= s0["cached"] + (4 << 20)
    q = lib.harp_host_malloc(4 << 20, 0, stream)  # same class: the cached block comes back
    assert q == p
    lib.harp_host_free(q, 4 << 20, 0, stream)
    alloc.empty_host_cache()
    assert alloc.stats("host")["cached"] == 0


def test_caps_fail_cleanly():
    from harp_b200.runtime import alloc

    alloc.set_cap("device", 4 << 20)
    try:
        with alloc.use_tier("device"):
            a = torch.empty(1 << 18, device="cuda", dtype=torch.float32)
            with pytest.raises(torch.OutOfMemoryError):
                torch.empty(16 << 20, device="cuda", dtype=torch.float32)
            del a
        assert alloc.stats("device")["failures"] >= 1
    finally:
        alloc.set_cap("device", 0)
