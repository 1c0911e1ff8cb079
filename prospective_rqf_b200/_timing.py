"""Optional CUDA-event timing of the backend's own kernel launches.

When a KernelTimer is active, each C-ABI call made by ops.py is bracketed by
CUDA events recorded on the launching stream (torch's current stream, which
is where the kernels run).  Used by bench.py and microbench.py to measure the
scan kernels' average launch duration inside timed work.  Each launch also
records its algorithmic bytes: the bytes of the large (per-sample) tensors it
must read and write once, counted from the tensors themselves; the per-tile
carries and per-filter coefficients are left out (below 0.1 %).
"""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch

_ACTIVE: "KernelTimer | None" = None


class KernelTimer:
    def __init__(self):
        self.events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = defaultdict(list)
        self.meta: dict[str, list[int]] = defaultdict(list)
        self.nbytes: dict[str, list[int]] = defaultdict(list)
        self.flops: dict[str, list[int]] = defaultdict(list)

    def __enter__(self):
        global _ACTIVE
        self._prev = _ACTIVE
        _ACTIVE = self
        return self

    def __exit__(self, *exc):
        global _ACTIVE
        _ACTIVE = self._prev
        return False

    def summary(self) -> dict[str, dict[str, float]]:
        """{name: {launches, total_ms, mean_ms, elements, alg_bytes}} (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for name, evs in self.events.items():
            ms = [a.elapsed_time(b) for a, b in evs]
            out[name] = {"launches": len(ms), "total_ms": float(sum(ms)),
                         "mean_ms": float(sum(ms) / max(len(ms), 1)),
                         "elements": int(sum(self.meta[name])),
                         "alg_bytes": int(sum(self.nbytes[name])),
                         "flops": int(sum(self.flops[name]))}
        return out


@contextmanager
def launch(name: str, elements: int, nbytes: int = 0, flops: int = 0):
    """Bracket one kernel launch (no-op unless a KernelTimer is active);
    `nbytes` = the launch's algorithmic bytes, `flops` its fp32-work FLOPs
    (GEMMs)."""
    t = _ACTIVE
    if t is None:
        yield
        return
    s = torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(s)
    yield
    b.record(s)
    t.events[name].append((a, b))
    t.meta[name].append(int(elements))
    t.nbytes[name].append(int(nbytes))
    t.flops[name].append(int(flops))
