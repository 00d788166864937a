"""Datasets: the reference's .npz sample format and synthetic data of the
benchmark shapes.

NpzDataset reads an index.json listing .npz files, each holding
`norm_metadata` [n_meta], `prompt_embeds` [L, cap_dim], `latent_image`
[C, H, W] and `cond` [C_cond, H, W] (the reference's
src/datatsets/TiffDataset.py:3-44, whose train.py imports it under other
names).  Paths in the index may be absolute or relative to the index file's
directory; a path whose leading directories do not exist is also tried by its
file name next to the index (the shipped index lists "HARP/data/...").

`collate` stacks metadata, latents and conditions and keeps the caption
embeddings as a list (captions may differ in length), giving `cond` as a list
with one stacked condition tensor, as the reference's custom_collate_fn does.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List

import numpy as np
import torch
from torch.utils.data import Dataset


class NpzDataset(Dataset):
    def __init__(self, index_path: str):
        if os.path.isdir(index_path):
            index_path = os.path.join(index_path, "index.json")
        with open(index_path) as fh:
            entries = json.load(fh)
        root = os.path.dirname(os.path.abspath(index_path))
        self.files = [self._resolve(e, root) for e in entries]
        first = np.load(self.files[0])
        self.num_metadata = int(first["norm_metadata"].shape[0]) if "norm_metadata" in first else 0

    @staticmethod
    def _resolve(path: str, root: str) -> str:
        for cand in (path, os.path.join(root, path), os.path.join(root, os.path.basename(path.replace("\\", "/")))):
            if os.path.exists(cand):
                return cand
        raise FileNotFoundError(f"sample {path} not found (index directory {root})")

    def __len__(self) -> int:
        return len(self.files)

    def __getitem__(self, idx: int) -> Dict[str, np.ndarray]:
        d = np.load(self.files[idx])
        return {k: d[k] for k in ("norm_metadata", "prompt_embeds", "latent_image", "cond") if k in d}


def collate(batch: List[Dict[str, np.ndarray]]) -> Dict[str, object]:
    out: Dict[str, object] = {}
    if "norm_metadata" in batch[0]:
        out["norm_metadata"] = torch.stack([torch.from_numpy(np.asarray(b["norm_metadata"])) for b in batch])
    out["prompt_embeds"] = [torch.from_numpy(np.asarray(b["prompt_embeds"])) for b in batch]
    out["latent_image"] = torch.stack([torch.from_numpy(np.asarray(b["latent_image"])) for b in batch])
    if "cond" in batch[0]:
        out["cond"] = [torch.stack([torch.from_numpy(np.asarray(b["cond"])) for b in batch])]
    return out


# reference names (train.py:36 imports these; the reference module defines NpzDataset/custom_collate_fn)
custom_collate_fn = collate
TiffDataset = NpzDataset
collate_fn = collate


class SyntheticDiTData(Dataset):
    """Random latents / caption embeddings of fixed shapes (benchmarks and tests:
    there is no network access for real data).  Deterministic per index."""

    def __init__(self, length: int, latent_channels: int, latent_size: int, text_len: int, text_dim: int,
                 num_metadata: int = 0, cond_channels: int = 0, seed: int = 0, dtype=torch.bfloat16):
        self.length, self.C, self.L = length, latent_channels, latent_size
        self.text_len, self.text_dim = text_len, text_dim
        self.num_metadata, self.cond_channels = num_metadata, cond_channels
        self.seed, self.dtype = seed, dtype

    def __len__(self):
        return self.length

    def __getitem__(self, idx):
        g = torch.Generator().manual_seed(self.seed * 1000003 + idx)
        item = {
            "latent_image": torch.randn(self.C, self.L, self.L, generator=g).to(self.dtype).numpy()
            if self.dtype == torch.float32 else torch.randn(self.C, self.L, self.L, generator=g).float().numpy(),
            "prompt_embeds": torch.randn(self.text_len, self.text_dim, generator=g).float().numpy(),
        }
        if self.num_metadata:
            item["norm_metadata"] = torch.rand(self.num_metadata, generator=g).float().numpy()
        if self.cond_channels:
            item["cond"] = torch.randn(self.cond_channels, self.L, self.L, generator=g).float().numpy()
        return item


def write_npz_samples(directory: str, n: int, latent_channels=16, latent_size=64, text_len=64, text_dim=2560,
                      num_metadata=4, cond_channels=192, seed=0) -> str:
    """Write `n` synthetic samples in the reference's .npz layout plus index.json
    (for tests and dry runs); returns the index path."""
    os.makedirs(directory, exist_ok=True)
    ds = SyntheticDiTData(n, latent_channels, latent_size, text_len, text_dim, num_metadata, cond_channels, seed,
                          dtype=torch.float32)
    names = []
    for i in range(n):
        p = os.path.join(directory, f"sample_{i:05d}.npz")
        np.savez(p, **ds[i])
        names.append(os.path.basename(p))
    idx = os.path.join(directory, "index.json")
    with open(idx, "w") as fh:
        json.dump(names, fh, indent=2)
    return idx
