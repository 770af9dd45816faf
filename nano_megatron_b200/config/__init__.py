"""Public configuration API (same names as the reference's nano_megatron.config)."""

from .loader import (
    ConfigLoadError,
    ConfigWarning,
    apply_override,
    config_from_dict,
    config_to_dict,
    load_config,
    load_config_with_result,
)
from .schema import (
    ActivationCheckpointConfig,
    ActivationCheckpointMode,
    CheckpointConfig,
    ContextParallelBackend,
    ContextParallelConfig,
    DataConfig,
    DataParallelConfig,
    DataParallelMode,
    DistributedConfig,
    GPTConfig,
    KernelBackend,
    KernelConfig,
    LearningRateSchedule,
    LearningRateSchedulerConfig,
    OffloadConfig,
    OptimizerConfig,
    ParallelConfig,
    PipelineConfig,
    PipelineSchedule,
    PrecisionConfig,
    PrecisionDType,
    TokenizerConfig,
    TrainConfig,
    TrainingConfig,
    ValidationConfig,
    WandbConfig,
)
from .validation import ConfigValidationError, ValidationResult, validate_config, validate_train_config

__all__ = [name for name in dir() if not name.startswith("_")]
