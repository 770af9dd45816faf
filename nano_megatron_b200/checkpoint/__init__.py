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

__all__ = [n for n in dir() if not n.startswith("_")]
