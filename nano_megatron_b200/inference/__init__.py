"""Checkpoint export to single-device artifacts and KV-cached generation."""

from .artifact import (
    ARTIFACT_NAME,
    ARTIFACT_VERSION,
    InferenceArtifact,
    InferenceArtifactError,
    export_checkpoint,
    load_inference_artifact,
)
from .generation import (
    GenerationResult,
    KVCacheDecoder,
    generate_from_artifact,
    generate_text,
    load_model_for_generation,
    sample_next_token,
)

__all__ = ["ARTIFACT_NAME", "ARTIFACT_VERSION", "GenerationResult", "InferenceArtifact",
           "InferenceArtifactError", "KVCacheDecoder", "export_checkpoint",
           "generate_from_artifact", "generate_text", "load_inference_artifact",
           "load_model_for_generation", "sample_next_token"]
