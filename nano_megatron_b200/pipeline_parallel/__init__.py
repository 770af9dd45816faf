"""Pipeline parallelism: partitioning, P2P transport and GPipe/1F1B/interleaved schedules."""

from .partition import (
    LayerPartition,
    PipelineStageAddress,
    VirtualPipelineLayout,
    partition_for_rank,
    partition_layers,
)

__all__ = [n for n in dir() if not n.startswith("_")]
