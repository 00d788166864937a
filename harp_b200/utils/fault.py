"""Host-side fault injection and failure detection.

Faults are injected on the host only (never by making a GPU fault or hang):
HARP_FAULT="<kind>@<site>[:<value>][,<kind>@<site>[:<value>]...]" with kinds
  raise      raise HarpInjectedFault when `site` is reached (value = step, or any)
  delay_ms   sleep `value` ms at `site` (a slow rank)
  exit       the rank exits with code 17 at `site` (value = step): a rank that
             leaves between steps, with nothing of its own in flight
  drop       skip the `site` action once (e.g. a signal that is never sent)
Sites used by the engine: "step" (start of a training step), "signal"
(an NVLink flag store), "grad_sync", "checkpoint".

Failure detection: device waits are bounded (the kernels record an error
word; harp_b200.runtime.errors raises HarpDeviceError), process-group
collectives get a short timeout, and Heartbeat publishes a per-rank counter
in the torch.distributed store so a rank can tell which peer stopped.
"""
from __future__ import annotations

import os
import sys
import threading
import time
from typing import Dict, List, Optional, Tuple


class HarpInjectedFault(RuntimeError):
    pass


class FaultInjector:
    def __init__(self, spec: Optional[str] = None, rank: int = 0):
        self.rank = rank
        self.rules: List[Tuple[str, str, Optional[str]]] = []
        spec = os.environ.get("HARP_FAULT", "") if spec is None else spec
        for part in filter(None, (p.strip() for p in spec.split(","))):
            kind, _, rest = part.partition("@")
            site, _, value = rest.partition(":")
            self.rules.append((kind, site, value or None))
        only = os.environ.get("HARP_FAULT_RANK")
        self.active = only is None or int(only) == rank

    def fire(self, site: str, step: Optional[int] = None) -> bool:
        """Apply rules for `site`; returns False when the action should be dropped."""
        if not self.active:
            return True
        keep = True
        for kind, s, value in list(self.rules):
            if s != site:
                continue
            if kind in ("raise", "exit") and value is not None and step is not None and int(value) != step:
                continue
            if kind == "raise":
                raise HarpInjectedFault(f"injected fault at {site} (step {step}, rank {self.rank})")
            if kind == "exit":
                sys.stdout.flush()
                os._exit(17)
            if kind == "delay_ms":
                time.sleep(float(value or 0) / 1000.0)
            if kind == "drop":
                self.rules.remove((kind, s, value))
                keep = False
        return keep


class Heartbeat:
    """Each rank bumps `harp/hb/<rank>` in the c10d store every `period_s`;
    `stale(timeout_s)` lists ranks whose counter has not moved."""

    def __init__(self, store, rank: int, world: int, period_s: float = 1.0):
        self.store, self.rank, self.world, self.period = store, rank, world, period_s
        self._stop = threading.Event()
        self._seen: Dict[int, Tuple[int, float]] = {}
        self._t = threading.Thread(target=self._run, daemon=True, name="harp-heartbeat")
        self._t.start()

    def _run(self):
        n = 0
        while not self._stop.is_set():
            n += 1
            try:
                self.store.set(f"harp/hb/{self.rank}", str(n))
            except Exception:
                return
            self._stop.wait(self.period)

    def stale(self, timeout_s: float) -> List[int]:
        now = time.time()
        out = []
        for r in range(self.world):
            try:
                v = int(self.store.get(f"harp/hb/{r}")) if self.store.check([f"harp/hb/{r}"]) else -1
            except Exception:
                v = -1
            last = self._seen.get(r)
            if last is None or last[0] != v:
                self._seen[r] = (v, now)
            elif now - last[1] > timeout_s:
                out.append(r)
        return out

    def stop(self):
        self._stop.set()
        self._t.join(timeout=2 * self.period)
