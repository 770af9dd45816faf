"""Pipeline parallelism: partitioning, P2P transport and GPipe/1F1B/interleaved schedules."""

from .partition import (
    LayerPartition,
    PipelineStageAddress,
    VirtualPipelineLayout,
    partition_for_rank,
    partition_layers,
)
from .p2p import P2PCommunicator
from .schedules.executor import PipelineScheduleExecutor
from .schedules.plans import (
    build_1f1b_plan,
    build_gpipe_plan,
    build_interleaved_plan,
    build_interleaved_schedule_table,
)

__all__ = [n for n in dir() if not n.startswith("_")]
