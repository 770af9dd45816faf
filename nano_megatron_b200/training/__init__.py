"""Training engine: trainer, LR schedule, batch routing, metrics."""

from .batch_router import BatchRouter, shard_batch_for_context_parallel
from .lr_scheduler import LearningRateScheduler
from .metrics import MetricStore, aggregate_loss_metrics
from .microbatches import global_batch_size, split_microbatches
from .metric_history import (
    METRIC_HISTORY_VERSION,
    JsonlMetricHistory,
    MetricHistoryRecord,
    read_metric_history,
)
from .trainer import Trainer, TrainerState
from .wandb_logger import WandbLogger

__all__ = [n for n in dir() if not n.startswith("_")]
