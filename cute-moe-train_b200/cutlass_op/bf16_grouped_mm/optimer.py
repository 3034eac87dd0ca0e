"""Optional per-operator device timing: CUDA events recorded on the current stream around every
grouped_mm operator call (forward wrappers and autograd backward alike).  Disabled by default;
when disabled each call costs one attribute check."""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch

_active: "OpTimer | None" = None


class OpTimer:
    """Collects (start, end) CUDA event pairs per operator name while installed."""

    def __init__(self) -> None:
        self.events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = defaultdict(list)

    def install(self) -> "OpTimer":
        global _active
        _active = self
        return self

    def uninstall(self) -> None:
        global _active
        if _active is self:
            _active = None

    def summary(self) -> dict[str, dict[str, float]]:
        """{name: {'launches': n, 'total_ms': t, 'avg_ms': t/n}} (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for name, pairs in self.events.items():
            ms = [a.elapsed_time(b) for a, b in pairs]
            out[name] = {"launches": len(ms), "total_ms": sum(ms), "avg_ms": sum(ms) / max(1, len(ms))}
        return out


@contextmanager
def timed(name: str):
    t = _active
    if t is None:
        yield
        return
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    try:
        yield
    finally:
        b.record()
        t.events[name].append((a, b))
