import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: test needs two or more GPUs")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _bounds_clean(request):
    """With HARP_DEBUG_BOUNDS=1 (the bounds-checking build), every GPU test
    must leave no recorded TMA-coordinate or tensor-memory-column violation."""
    yield
    if os.environ.get("HARP_DEBUG_BOUNDS") != "1" or "gpu" not in request.keywords:
        return
    import torch

    if not torch.cuda.is_available() or not hasattr(torch.ops, "harp") or not hasattr(torch.ops.harp,
                                                                                       "debug_bounds_status"):
        return
    st = torch.ops.harp.debug_bounds_status().tolist()
    assert st[4] > 0, "HARP_DEBUG_BOUNDS=1 but the loaded library has no bounds checks compiled in"
    assert st[0] == 0, f"bounds violation {st[:4]} (code, site, block, info)"
