"""The reference's import paths, for code written against it.

The reference's scripts import its modules by top-level names:
`from managers.shard_manager import SequenceScatter`,
`from async_rt.runtime import AsyncSync`, `from unigemm_linear import kpLinear`,
`from kp_rope_embedder import replace_ropeembedder_with_sverope`, and so on
(train.py:36-66, src/models/z_image/hl_model.py:6-24, module/attn.py:9-12).
`install_reference_import_paths()` registers each of those names in
`sys.modules` as the harp module that implements it, so that such code runs
unchanged afterwards:

    import harp_b200.compat
    harp_b200.compat.install_reference_import_paths()
    from managers.weight_manager import build_chunk_param   # harp_b200.managers.weight_manager

A name that already resolves to a module of another origin (for example the
reference's own package on sys.path, already imported) is left alone, with
its submodules, unless `replace=True`.  `python -m harp_b200.compat` prints the table.
"""
from __future__ import annotations

import importlib
import sys
from typing import Dict, List

# reference import path -> harp module that implements it
REFERENCE_MODULES: Dict[str, str] = {
    "managers": "harp_b200.managers",
    "managers.shard_manager": "harp_b200.managers.shard_manager",
    "managers.weight_manager": "harp_b200.managers.weight_manager",
    "managers.grad_manager": "harp_b200.managers.grad_manager",
    "managers.mem_manager": "harp_b200.managers.mem_manager",
    "managers.ring_attn_manager": "harp_b200.managers.ring_attn_manager",
    "async_rt": "harp_b200.runtime.async_compat",
    "async_rt.runtime": "harp_b200.runtime.async_compat",
    "async_rt.async_ops": "harp_b200.runtime.async_compat",
    "unigemm_linear": "harp_b200.ops.modules",
    "kp_normalization": "harp_b200.ops.modules",
    "kp_multi_tensor_adamw": "harp_b200.ops.modules",
    "kp_rope": "harp_b200.ops.modules",
    "kp_rope_embedder": "harp_b200.models.zimage",
}


def install_reference_import_paths(replace: bool = False) -> List[str]:
    """Register the reference's module names; returns the names registered."""
    done, kept = [], set()
    for name, target in REFERENCE_MODULES.items():
        mod = importlib.import_module(target)
        cur = sys.modules.get(name)
        parent = name.rpartition(".")[0]
        if not replace and (parent in kept or (cur is not None and cur is not mod)):
            kept.add(name)  # another package of this name is in use: leave its subtree alone
            continue
        sys.modules[name] = mod
        parent, _, child = name.rpartition(".")
        if parent:  # `from async_rt import async_ops` reads the attribute first
            setattr(sys.modules[parent], child, mod)
        done.append(name)
    return done


if __name__ == "__main__":
    w = max(map(len, REFERENCE_MODULES))
    for k, v in REFERENCE_MODULES.items():
        print(f"{k:<{w}}  {v}")
