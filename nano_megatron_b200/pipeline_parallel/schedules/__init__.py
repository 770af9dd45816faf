"""Pipeline schedules (GPipe, 1F1B, interleaved 1F1B) and the executor."""

from .base import LossAccumulator, extract_loss
from .executor import PipelineScheduleExecutor
from .no_pipeline import NoPipelineSchedule
from .plans import (
    build_1f1b_plan,
    build_gpipe_plan,
    build_interleaved_plan,
    build_interleaved_schedule_table,
)


def build_schedule(config, model, parallel, data_parallel):
    if parallel.pp.size == 1 and config.pipeline.virtual_stages_per_rank == 1:
        from nano_megatron_b200.training.cuda_graphs import graphs_supported

        device = next(model.parameters()).device
        return NoPipelineSchedule(model, data_parallel,
                                  use_graphs=graphs_supported(config, model, data_parallel,
                                                              device))
    from .executor import build_pipeline_schedule

    return build_pipeline_schedule(config, model, parallel, data_parallel)


__all__ = ["LossAccumulator", "NoPipelineSchedule", "PipelineScheduleExecutor",
           "build_1f1b_plan", "build_gpipe_plan", "build_interleaved_plan",
           "build_interleaved_schedule_table", "build_schedule", "extract_loss"]
