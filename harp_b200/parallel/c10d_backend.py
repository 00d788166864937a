"""Register the harp_nvl NVLink backend with torch.distributed.

    from harp_b200.parallel import c10d_backend
    c10d_backend.register()                          # once per process
    dist.init_process_group("cpu:gloo,cuda:harp_nvl")  # or dist.new_group(backend="harp_nvl")

The backend (csrc/c10d_nvl.cpp) is the B200 counterpart of the reference's
HMPI process group (hmpi/ProcessGroupHMPI.cpp:50-76 registers it the same
way, under "hmpi" for CPU tensors): collectives of CUDA tensors on the GPUs of
one node, run as harp kernels over NVLink peer memory on the caller's stream.
"""
from __future__ import annotations

import torch.distributed as dist

from .. import _native

NAME = "harp_nvl"
_registered = set()


def register(name: str = NAME) -> str:
    if name in _registered:
        return name
    mod = _native.load_c10d()

    def _create(store, rank, size, timeout):
        return mod.create_backend(store, rank, size, timeout)

    dist.Backend.register_backend(name, _create, devices=["cuda"])
    _registered.add(name)
    return name
