"""Tracing hooks: NVTX ranges and a torch.profiler window over chosen training steps.

* ``nvtx_range(name)`` pushes an NVTX range around host code when ``NMB_NVTX=1`` (and CUDA
  is available), so Nsight Systems timelines show steps, microbatches, pipeline actions
  and transformer blocks by name; otherwise it costs one dictionary lookup. Ranges are
  host-side markers: inside a captured CUDA graph they mark the capture, not replays.
* ``StepProfiler`` runs ``torch.profiler`` (CPU + CUDA activities) for steps
  ``[start, stop)`` and writes one Chrome trace per rank into a directory.

The reference has neither (profiling lives only in its GPU tests); device-timed
tokens/s and per-phase step times come from ``utils.timing.StepPhaseTimer``.
"""

from __future__ import annotations

import os
from contextlib import contextmanager, nullcontext
from pathlib import Path

import torch

_ENABLED: bool | None = None


def nvtx_enabled() -> bool:
    global _ENABLED
    if _ENABLED is None:
        _ENABLED = os.environ.get("NMB_NVTX", "0") == "1" and torch.cuda.is_available()
    return _ENABLED


@contextmanager
def _nvtx(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_range(name: str):
    return _nvtx(name) if nvtx_enabled() else nullcontext()


class StepProfiler:
    """Profile training steps ``start <= step < stop``; one trace file per rank."""

    def __init__(self, directory, start: int, stop: int, rank: int = 0) -> None:
        if not 0 <= start < stop:
            raise ValueError("profile steps must satisfy 0 <= start < stop")
        self.directory = Path(directory)
        self.start, self.stop, self.rank = int(start), int(stop), int(rank)
        self._prof = None
        self.trace_path: Path | None = None

    def before_step(self, step: int) -> None:
        if step == self.start and self._prof is None:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self._prof = torch.profiler.profile(activities=acts, record_shapes=False,
                                                acc_events=True)
            self._prof.__enter__()

    def after_step(self, step: int) -> None:
        """``step`` = the number of completed steps after this one."""
        if self._prof is not None and step >= self.stop:
            self._prof.__exit__(None, None, None)
            self.directory.mkdir(parents=True, exist_ok=True)
            self.trace_path = self.directory / f"trace_rank{self.rank:04d}.json"
            self._prof.export_chrome_trace(str(self.trace_path))
            self._prof = None

    def close(self) -> None:
        if self._prof is not None:
            self.after_step(self.stop)
