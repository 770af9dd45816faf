"""Device-side step timing: CUDA events on the launching stream, max over ranks."""

from __future__ import annotations

import time

import torch
import torch.distributed as dist


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


def max_over_ranks(value: float, device: torch.device, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
