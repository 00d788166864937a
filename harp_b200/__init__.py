"""harp_b200: a Blackwell-native (sm_100a) sequence-parallel DiT training framework.

Capabilities follow wxyww2049/HARP (ring-attention sequence parallelism,
intra-node weight/gradient sharing, optimizer-state sharding with asynchronous
parameter all-gather, the managers/ API), re-designed for 8xB200: PyTorch for
the framework layer, hand-written tcgen05/TMA CUDA kernels for the hot ops,
NVLink peer memory for the fused collectives.
"""
from . import _native  # noqa: F401

__version__ = "0.1.0"


def load_native(build_if_needed: bool = False) -> bool:
    """Load the CUDA library (harp_b200/_build/harp_b200_C.so)."""
    return _native.load(build_if_needed=build_if_needed)
