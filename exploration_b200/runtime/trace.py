"""Tracing hooks: NVTX phase ranges and a torch.profiler window.

* ``phase(name)``: an NVTX range around a phase of a step (encode, read
  rounds, head, backward, gradient reduction, optimizer) when ``EB200_NVTX=1``
  (or while ``profile_steps`` records); free otherwise. The ranges show up in
  any CUDA timeline tool.
* ``profile_steps(directory, rank)``: a torch.profiler session over a few
  training steps (1 skipped, 1 warm-up, 3 recorded) that writes a Chrome
  trace per rank and returns the kernel summary for the JSONL log.

The reference has phase timers on the model (st/models/stack.py:385-460) and
no profiler integration.
"""
from __future__ import annotations

import contextlib
import os
from pathlib import Path

import torch

_force = False


def enabled() -> bool:
    return _force or os.environ.get("EB200_NVTX", "0") == "1"


@contextlib.contextmanager
def phase(name: str):
    if not (enabled() and torch.cuda.is_available()):
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class StepProfiler:
    """Call ``step()`` after every training step; ``summary()`` after the loop."""

    def __init__(self, directory: str, rank: int = 0, wait: int = 1, warmup: int = 1, active: int = 3):
        global _force
        self.path = Path(directory)
        self.path.mkdir(parents=True, exist_ok=True)
        self.rank = rank
        activities = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(torch.profiler.ProfilerActivity.CUDA)
        self.prof = torch.profiler.profile(
            activities=activities,
            schedule=torch.profiler.schedule(wait=wait, warmup=warmup, active=active, repeat=1),
            on_trace_ready=self._ready)
        self.table = None
        _force = True
        self.prof.__enter__()

    def _ready(self, prof):
        prof.export_chrome_trace(str(self.path / f"trace_rank{self.rank}.json"))
        device = "cuda" if torch.cuda.is_available() else "cpu"
        key = f"self_{device}_time_total"
        rows = []
        for event in prof.key_averages():
            rows.append({"name": event.key[:120], "calls": event.count,
                         "self_us": round(float(getattr(event, key, 0.0)), 1)})
        rows.sort(key=lambda r: -r["self_us"])
        self.table = rows[:25]

    def step(self):
        self.prof.step()

    def summary(self):
        global _force
        self.prof.__exit__(None, None, None)
        _force = False
        return {"trace": str(self.path / f"trace_rank{self.rank}.json"), "top": self.table or []}
