"""Checkpoint save/resume in the reference's on-disk layout (manifest schema 2)."""

from .manager import CheckpointManager, capture_runtime_state, restore_runtime_state
from .manifest import (
    SCHEMA_VERSION,
    CheckpointManifest,
    RankLocalShard,
    RankRuntimeState,
    ShardMetadata,
    make_manifest,
    validate_topology,
)
from .mapping import ShardedState, infer_shard_metadata, iter_tensors

__all__ = [n for n in dir() if not n.startswith("_")] + ["TrainerState"]


def __getattr__(name: str):
    # TrainerState (what a checkpoint's trainer entry restores) lives with the trainer;
    # imported on first use, since the trainer imports this package
    if name == "TrainerState":
        from nano_megatron_b200.training.trainer import TrainerState

        return TrainerState
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
