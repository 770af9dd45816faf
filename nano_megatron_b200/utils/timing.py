"""Device-side step timing: CUDA events on the launching stream, max over ranks.

:class:`StepPhaseTimer` marks the boundaries of one training step's phases
(forward+backward, gradient synchronisation, clipping, optimizer) with CUDA events
and resolves them only when asked, so timing adds no host synchronisation to the
step loop; on CPU the marks are ``perf_counter`` readings. The reference times
throughput with the host clock over the log interval only
(src/nano_megatron/training/trainer.py:609-624).
"""

from __future__ import annotations

import time

import torch
import torch.distributed as dist

PHASES = ("forward_backward", "grad_sync", "clip", "optimizer")


class DeviceStepTimer:
    """Times a region with CUDA events (host ``perf_counter`` on CPU)."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.cuda = device.type == "cuda"

    def start(self) -> None:
        if self.cuda:
            self._s = torch.cuda.Event(enable_timing=True)
            self._e = torch.cuda.Event(enable_timing=True)
            self._s.record()
        else:
            self._t0 = time.perf_counter()

    def stop(self) -> None:
        if self.cuda:
            self._e.record()
        else:
            self._t1 = time.perf_counter()

    def elapsed_ms(self) -> float:
        if self.cuda:
            self._e.synchronize()
            return float(self._s.elapsed_time(self._e))
        return (self._t1 - self._t0) * 1000.0


class StepMarks:
    """The boundary marks of one step: ``start`` followed by one mark per finished phase."""

    def __init__(self, cuda: bool) -> None:
        self.cuda = cuda
        self.names: list[str] = []
        self.marks: list = []

    def add(self, name: str) -> None:
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append(ev)
        else:
            self.marks.append(time.perf_counter())
        self.names.append(name)

    def resolve(self) -> dict[str, float]:
        """Milliseconds per phase plus ``step``; waits for the step's last event."""
        if len(self.marks) < 2:
            return {}
        if self.cuda:
            self.marks[-1].synchronize()
            d = [float(a.elapsed_time(b)) for a, b in zip(self.marks, self.marks[1:])]
            total = float(self.marks[0].elapsed_time(self.marks[-1]))
        else:
            d = [(b - a) * 1000.0 for a, b in zip(self.marks, self.marks[1:])]
            total = (self.marks[-1] - self.marks[0]) * 1000.0
        out = dict(zip(self.names[1:], d))
        out["step"] = total
        return out


class StepPhaseTimer:
    """Creates :class:`StepMarks` for successive steps on ``device``."""

    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda"
        self.current: StepMarks | None = None

    def begin(self) -> None:
        self.current = StepMarks(self.cuda)
        self.current.add("start")

    def mark(self, phase: str) -> None:
        if self.current is not None:
            self.current.add(phase)

    def end(self) -> StepMarks | None:
        marks, self.current = self.current, None
        return marks


def summarize_phases(steps: list[StepMarks], device: torch.device, group=None) -> dict[str, float]:
    """Total milliseconds per phase (and ``step``) over ``steps``, max over ranks per phase."""
    keys = PHASES + ("step",)
    tot = dict.fromkeys(keys, 0.0)
    for m in steps:
        for k, v in m.resolve().items():
            if k in tot:
                tot[k] += v
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([tot[k] for k in keys], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        tot = dict(zip(keys, t.tolist()))
    return tot


def max_over_ranks(value: float, device: torch.device, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
