"""CUDA-event stage timer.

Records a start/stop event pair around named stages of one step on the
current stream and resolves them after a synchronize, so per-stage GPU time
can be read without a profiler.  Disabled timers cost nothing; graph capture
must not run with a timer enabled (events would be captured).

Reference counterpart: StageTimer / StageMs (engines/glm5-moe-nvfp4-2b/src/
model.cu:41-71, model.h:55-77), enabled only on the instrumented step.
"""
from __future__ import annotations

from collections import defaultdict

import torch


class StageTimer:
    """`enabled`: CUDA-event pairs per stage.  `nvtx`: NVTX ranges with the stage names
    (host-side markers for an external timeline profiler; safe during graph capture)."""

    def __init__(self, enabled: bool = False, nvtx: bool = False):
        self.enabled = enabled
        self.nvtx = nvtx
        self._open: dict[str, torch.cuda.Event] = {}
        self._pairs: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self, name: str):
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[name] = e

    def stop(self, name: str):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._pairs.append((name, self._open.pop(name), e))
        if self.nvtx:
            torch.cuda.nvtx.range_pop()

    class _Span:
        def __init__(self, t, name):
            self.t, self.name = t, name

        def __enter__(self):
            self.t.start(self.name)

        def __exit__(self, *a):
            self.t.stop(self.name)

    def span(self, name: str):
        return StageTimer._Span(self, name)

    def resolve(self) -> dict[str, float]:
        """Synchronize and return summed milliseconds per stage; clears the record."""
        if not self._pairs:
            return {}
        torch.cuda.synchronize()
        out: dict[str, float] = defaultdict(float)
        for name, a, b in self._pairs:
            out[name] += a.elapsed_time(b)
        self._pairs.clear()
        return dict(out)


NULL_TIMER = StageTimer(False)
