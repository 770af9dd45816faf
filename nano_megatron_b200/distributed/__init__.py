"""Process-group runtime and the symmetric-memory layer for fused collectives."""

from .runtime import DistributedRuntime, DistributedRuntimeError, DistributedUnavailableError

__all__ = ["DistributedRuntime", "DistributedRuntimeError", "DistributedUnavailableError"]
