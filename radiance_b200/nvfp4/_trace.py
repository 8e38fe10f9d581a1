"""Optional per-launch timing of the library's kernels (CUDA events on the launching stream).

Inactive by default: each op checks one module global.  ``with kernel_timer() as kt:`` records a
start/end event pair around every C-ABI launch, with the launch's algorithmic work (FLOPs for a
GEMM, bytes for a quantizer or amax pass), so a caller can report per-kind device time and
throughput without a profiler.  The events are created "external", so a step captured in a CUDA
graph under the timer keeps them as event-record nodes: every replay re-records them, and
``summary()`` after a replay gives that replay's per-launch times.
"""

from __future__ import annotations

import contextlib
from collections import defaultdict

import torch


class KernelTimer:
    def __init__(self) -> None:
        self.records: list[tuple[str, float, torch.cuda.Event, torch.cuda.Event]] = []
        self.launches = 0

    def summary(self) -> dict[str, dict[str, float]]:
        """Per kind: launches, total device ms, total work (FLOPs or bytes).  Synchronises."""
        torch.cuda.synchronize()
        out: dict[str, dict[str, float]] = defaultdict(lambda: {"launches": 0, "ms": 0.0, "work": 0.0})
        for kind, work, s, e in self.records:
            d = out[kind]
            d["launches"] += 1
            d["ms"] += s.elapsed_time(e)
            d["work"] += work
        return dict(out)


_active: KernelTimer | None = None


@contextlib.contextmanager
def kernel_timer():
    global _active
    prev, _active = _active, KernelTimer()
    try:
        yield _active
    finally:
        _active = prev


def begin(kind: str, work: float):
    if _active is None:
        return None
    _active.launches += 1
    s = torch.cuda.Event(enable_timing=True, external=True)
    s.record()
    return (kind, work, s)


def end(token) -> None:
    if token is None or _active is None:
        return
    e = torch.cuda.Event(enable_timing=True, external=True)
    e.record()
    _active.records.append((token[0], token[1], token[2], e))
