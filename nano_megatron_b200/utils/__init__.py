"""Small shared utilities (device timing, NVTX ranges)."""

from .timing import DeviceStepTimer, StepPhaseTimer, max_over_ranks, summarize_phases

__all__ = ["DeviceStepTimer", "StepPhaseTimer", "max_over_ranks", "summarize_phases"]
