"""Device error words.

Every waiting kernel of the library takes a 4-int32 error word: a wait that
runs out of time records {code, site, block, info} there and returns instead
of spinning on (see csrc/common.cuh).  The host reads the word after a step
(:func:`check`) and raises :class:`HarpDeviceError`, leaving the CUDA context
usable.
"""
from __future__ import annotations

import threading
from typing import Dict

import torch

CODES = {0: "ok", 1: "pipeline wait timeout", 2: "peer/flag wait timeout", 3: "bounds check"}

_lock = threading.Lock()
_words: Dict[int, torch.Tensor] = {}


class HarpDeviceError(RuntimeError):
    def __init__(self, code: int, site: int, block: int, info: int):
        self.code, self.site, self.block, self.info = code, site, block, info
        super().__init__(
            f"harp device error: {CODES.get(code, code)} at site {site} (block {block}, info {info})"
        )


def word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _words.get(idx)
    if w is None:
        with _lock:
            w = _words.get(idx)
            if w is None:
                w = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
                _words[idx] = w
    return w


def check(device=None, clear: bool = True) -> None:
    """Raise HarpDeviceError if any kernel on `device` recorded an error (syncs)."""
    if not torch.cuda.is_available():
        return
    devs = [device] if device is not None else [torch.device("cuda", i) for i in list(_words)]
    for d in devs:
        w = word(torch.device(d) if not isinstance(d, torch.device) else d)
        vals = w.cpu().tolist()
        if vals[0] != 0:
            if clear:
                w.zero_()
            raise HarpDeviceError(*vals)
