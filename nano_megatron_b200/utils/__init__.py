"""Small shared utilities (device timing, NVTX ranges)."""

from .timing import DeviceStepTimer, max_over_ranks

__all__ = ["DeviceStepTimer", "max_over_ranks"]
