"""Typed configuration blocks.

The YAML schema is the reference's (src/nano_megatron/config/schema.py:60-665):
the same 17 blocks, field names, defaults and per-field checks, so reference
YAML files load unchanged. Additions are strictly additive:

* ``kernels.backend`` also accepts ``b200``; every value selects this library's
  sm_100a kernels on CUDA devices (``torch`` is kept as a compatible spelling).
* ``kernels.cuda_graphs`` captures the per-microbatch forward/backward of
  static-shape runs in CUDA graphs.
* ``kernels.fused_tp_comm`` / ``fused_dp_comm`` / ``fused_cp_comm`` select the
  collectives fused over NVLink peer memory, and ``kernels.deterministic`` the
  fixed-order (bitwise reproducible) backward reductions.
* ``context_parallel.load_balance`` selects zigzag chunking (rank r holds
  sequence chunks r and 2*CP-1-r) instead of contiguous chunks.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import StrEnum
from pathlib import Path

from nano_megatron_b200.parallel.axes import DEFAULT_RANK_ORDER, ParallelAxis, normalize_rank_order


# ------------------------------------------------------------------ field checks
def _int(name: str, value, minimum: int = 1) -> None:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be an integer, got {value!r}")
    if value < minimum:
        raise ValueError(f"{name} must be >= {minimum}, got {value}")


def _bool(name: str, value) -> None:
    if not isinstance(value, bool):
        raise TypeError(f"{name} must be a boolean, got {value!r}")


def _number(name: str, value, *, allow_zero: bool = False) -> None:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{name} must be a number, got {value!r}")
    if value < 0 or (value == 0 and not allow_zero):
        raise ValueError(f"{name} must be {'>=' if allow_zero else '>'} 0, got {value}")


def _path(name: str, value) -> Path | None:
    if value is None:
        return None
    if not isinstance(value, (str, Path)):
        raise TypeError(f"{name} must be a filesystem path string or null")
    if isinstance(value, str) and not value.strip():
        raise ValueError(f"{name} must not be empty")
    return Path(value)


def _enum(name: str, kind: type[StrEnum], value):
    try:
        return kind(value)
    except (TypeError, ValueError) as error:
        choices = ", ".join(m.value for m in kind)
        raise ValueError(f"{name} must be one of: {choices}; got {value!r}") from error


def _set(obj, name: str, value) -> None:
    object.__setattr__(obj, name, value)


# ------------------------------------------------------------------ enums
class PrecisionDType(StrEnum):
    FLOAT32 = "float32"
    BFLOAT16 = "bfloat16"
    FLOAT16 = "float16"


class KernelBackend(StrEnum):
    TORCH = "torch"
    B200 = "b200"


class DataParallelMode(StrEnum):
    DDP = "ddp"
    ZERO1 = "zero1"
    ZERO2 = "zero2"
    ZERO3 = "zero3"


class PipelineSchedule(StrEnum):
    ONE_F_ONE_B = "1f1b"
    GPIPE = "gpipe"
    INTERLEAVED_ONE_F_ONE_B = "interleaved_1f1b"


class ContextParallelBackend(StrEnum):
    ALL_GATHER = "all_gather"
    RING = "ring"


class ActivationCheckpointMode(StrEnum):
    NONE = "none"
    FULL = "full"
    SELECTIVE = "selective"


class LearningRateSchedule(StrEnum):
    CONSTANT = "constant"
    COSINE = "cosine"


# ------------------------------------------------------------------ blocks
@dataclass(frozen=True, slots=True)
class DistributedConfig:
    backend: str = "auto"
    timeout_minutes: int = 30
    device: str = "auto"
    init_method: str = "env://"

    def __post_init__(self) -> None:
        for name in ("backend", "device", "init_method"):
            value = getattr(self, name)
            if not isinstance(value, str) or not value.strip():
                raise ValueError(f"distributed.{name} must be a non-empty string")
        _int("distributed.timeout_minutes", self.timeout_minutes)
        _set(self, "backend", self.backend.strip().lower())
        _set(self, "device", self.device.strip().lower())
        _set(self, "init_method", self.init_method.strip())


@dataclass(frozen=True, slots=True)
class ParallelConfig:
    tensor: int = 1
    pipeline: int = 1
    context: int = 1
    expert: int = 1
    data: int | None = None
    order: tuple[ParallelAxis, ...] = DEFAULT_RANK_ORDER
    sequence_parallel: bool = False

    def __post_init__(self) -> None:
        for name in ("tensor", "pipeline", "context", "expert"):
            _int(f"parallel.{name}", getattr(self, name))
        if self.data is not None:
            _int("parallel.data", self.data)
        _bool("parallel.sequence_parallel", self.sequence_parallel)
        _set(self, "order", normalize_rank_order(self.order))

    tensor_parallel_size = property(lambda self: self.tensor)
    pipeline_parallel_size = property(lambda self: self.pipeline)
    context_parallel_size = property(lambda self: self.context)
    expert_parallel_size = property(lambda self: self.expert)

    @property
    def data_parallel_size(self) -> int:
        if self.data is None:
            raise ValueError("parallel.data has not been resolved against a world size")
        return self.data

    @property
    def model_parallel_size(self) -> int:
        return self.tensor * self.pipeline * self.context * self.expert

    @property
    def configured_world_size(self) -> int | None:
        return None if self.data is None else self.model_parallel_size * self.data

    def resolve_data_parallel_size(self, world_size: int | None) -> int:
        if world_size is not None:
            _int("world_size", world_size)
        mp = self.model_parallel_size
        if self.data is not None:
            if world_size is not None and mp * self.data != world_size:
                raise ValueError(
                    "world size does not match parallel topology: "
                    f"{world_size} != TP({self.tensor}) * PP({self.pipeline}) * "
                    f"CP({self.context}) * EP({self.expert}) * DP({self.data}) = {mp * self.data}"
                )
            return self.data
        if world_size is None:
            raise ValueError("world_size is required when parallel.data is null")
        if world_size % mp:
            raise ValueError(f"world size {world_size} is not divisible by TP*PP*CP*EP ({mp})")
        return world_size // mp

    def resolved(self, world_size: int) -> "ParallelConfig":
        return ParallelConfig(self.tensor, self.pipeline, self.context, self.expert,
                              self.resolve_data_parallel_size(world_size), self.order,
                              self.sequence_parallel)


@dataclass(frozen=True, slots=True)
class GPTConfig:
    layers: int = 12
    hidden_size: int = 768
    ffn_hidden_size: int = 2048
    heads: int = 12
    kv_heads: int | None = None
    seq_length: int = 2048
    vocab_size: int = 50304
    rope_theta: float = 10000.0
    dropout: float = 0.0
    tie_embeddings: bool = True
    norm_epsilon: float = 1.0e-5
    bias: bool = False

    def __post_init__(self) -> None:
        for name in ("layers", "hidden_size", "ffn_hidden_size", "heads", "seq_length",
                     "vocab_size"):
            _int(f"model.{name}", getattr(self, name))
        if self.kv_heads is not None:
            _int("model.kv_heads", self.kv_heads)
        _number("model.rope_theta", self.rope_theta)
        _number("model.norm_epsilon", self.norm_epsilon)
        d = self.dropout
        if isinstance(d, bool) or not isinstance(d, (int, float)) or not 0 <= d < 1:
            raise ValueError(f"model.dropout must be in [0, 1), got {d}")
        _bool("model.tie_embeddings", self.tie_embeddings)
        _bool("model.bias", self.bias)
        if self.hidden_size % self.heads:
            raise ValueError(f"model.hidden_size ({self.hidden_size}) must be divisible by "
                             f"model.heads ({self.heads})")
        kv = self.num_kv_heads
        if kv > self.heads or self.heads % kv:
            raise ValueError("model.kv_heads must divide model.heads and cannot exceed it; "
                             f"got heads={self.heads}, kv_heads={kv}")

    num_layers = property(lambda self: self.layers)
    num_attention_heads = property(lambda self: self.heads)
    num_kv_heads = property(lambda self: self.heads if self.kv_heads is None else self.kv_heads)
    head_dim = property(lambda self: self.hidden_size // self.heads)

    def padded_vocab_size(self, tensor_parallel_size: int) -> int:
        _int("tensor_parallel_size", tensor_parallel_size)
        tp = tensor_parallel_size
        return -(-self.vocab_size // tp) * tp


@dataclass(frozen=True, slots=True)
class PrecisionConfig:
    params: PrecisionDType = PrecisionDType.BFLOAT16
    compute: PrecisionDType = PrecisionDType.BFLOAT16
    grad_reduce: PrecisionDType = PrecisionDType.FLOAT32

    def __post_init__(self) -> None:
        for name in ("params", "compute", "grad_reduce"):
            _set(self, name, _enum(f"precision.{name}", PrecisionDType, getattr(self, name)))


@dataclass(frozen=True, slots=True)
class KernelConfig:
    backend: KernelBackend = KernelBackend.TORCH
    cuda_graphs: bool = True
    # Sequence-parallel TP collectives fused into the GEMMs over NVLink symmetric memory
    # (AG->GEMM, GEMM->RS); off = NCCL all-gather / reduce-scatter around plain GEMMs.
    fused_tp_comm: bool = True
    # Data-parallel gradient reduction fused with the sharded AdamW update and the bf16
    # parameter all-gather over NVLink peer memory (DDP, ZeRO-1/2); off = NCCL collectives.
    fused_dp_comm: bool = True
    # Context-parallel ring attention pulling the next K/V block straight from its owner's
    # memory (peer loads) instead of NCCL send/recv.
    fused_cp_comm: bool = True
    # Fixed-order reductions in every backward kernel that otherwise sums with fp32
    # atomics (split-K weight gradients, attention dQ, RMSNorm dgamma, embedding backward):
    # bitwise reproducible steps at some speed cost.
    deterministic: bool = False

    def __post_init__(self) -> None:
        _set(self, "backend", _enum("kernels.backend", KernelBackend, self.backend))
        _bool("kernels.cuda_graphs", self.cuda_graphs)
        _bool("kernels.fused_tp_comm", self.fused_tp_comm)
        _bool("kernels.fused_dp_comm", self.fused_dp_comm)
        _bool("kernels.fused_cp_comm", self.fused_cp_comm)
        _bool("kernels.deterministic", self.deterministic)


@dataclass(frozen=True, slots=True)
class DataParallelConfig:
    mode: DataParallelMode = DataParallelMode.DDP
    bucket_bytes: int = 256 * 1024 * 1024
    overlap_grad_reduce: bool = False
    reshard_after_forward: bool = True

    def __post_init__(self) -> None:
        _set(self, "mode", _enum("data_parallel.mode", DataParallelMode, self.mode))
        _int("data_parallel.bucket_bytes", self.bucket_bytes)
        _bool("data_parallel.overlap_grad_reduce", self.overlap_grad_reduce)
        _bool("data_parallel.reshard_after_forward", self.reshard_after_forward)


@dataclass(frozen=True, slots=True)
class PipelineConfig:
    schedule: PipelineSchedule = PipelineSchedule.ONE_F_ONE_B
    activation_dtype: PrecisionDType | None = None
    overlap_p2p: bool = False
    virtual_stages_per_rank: int = 1
    dynamic_activation_shapes: bool = False

    def __post_init__(self) -> None:
        _set(self, "schedule", _enum("pipeline.schedule", PipelineSchedule, self.schedule))
        if self.activation_dtype is not None:
            _set(self, "activation_dtype",
                 _enum("pipeline.activation_dtype", PrecisionDType, self.activation_dtype))
        _bool("pipeline.overlap_p2p", self.overlap_p2p)
        _int("pipeline.virtual_stages_per_rank", self.virtual_stages_per_rank)
        _bool("pipeline.dynamic_activation_shapes", self.dynamic_activation_shapes)


@dataclass(frozen=True, slots=True)
class ContextParallelConfig:
    backend: ContextParallelBackend = ContextParallelBackend.ALL_GATHER
    dropout: float = 0.0
    load_balance: bool = False

    def __post_init__(self) -> None:
        _set(self, "backend", _enum("context_parallel.backend", ContextParallelBackend,
                                    self.backend))
        if isinstance(self.dropout, bool) or not isinstance(self.dropout, (int, float)):
            raise TypeError("context_parallel.dropout must be a number")
        if self.dropout != 0.0:
            raise ValueError("context_parallel.dropout must be 0 in phase one; CP attention "
                             "dropout is not implemented")
        _bool("context_parallel.load_balance", self.load_balance)


@dataclass(frozen=True, slots=True)
class ActivationCheckpointConfig:
    mode: ActivationCheckpointMode = ActivationCheckpointMode.NONE
    block_interval: int = 1
    selective_ops: tuple[str, ...] = ("attention", "mlp")
    use_reentrant: bool = False
    offload_saved_tensors: bool = False

    def __post_init__(self) -> None:
        _set(self, "mode", _enum("activation_checkpoint.mode", ActivationCheckpointMode, self.mode))
        _set(self, "selective_ops", tuple(self.selective_ops))
        _int("activation_checkpoint.block_interval", self.block_interval)
        if not self.selective_ops:
            raise ValueError("activation_checkpoint.selective_ops cannot be empty")
        unknown = sorted(set(self.selective_ops) - {"attention", "mlp"})
        if unknown:
            raise ValueError("activation_checkpoint.selective_ops contains unsupported values: "
                             + ", ".join(unknown))
        _bool("activation_checkpoint.use_reentrant", self.use_reentrant)
        if self.use_reentrant:
            raise ValueError("Nano-Megatron only supports non-reentrant activation checkpointing")
        _bool("activation_checkpoint.offload_saved_tensors", self.offload_saved_tensors)


@dataclass(frozen=True, slots=True)
class OffloadConfig:
    optimizer_state: bool = False
    zero3_params_and_grads: bool = False
    activations: bool = False
    pin_memory: bool = True
    non_blocking: bool = True

    def __post_init__(self) -> None:
        for name in ("optimizer_state", "zero3_params_and_grads", "activations", "pin_memory",
                     "non_blocking"):
            _bool(f"offload.{name}", getattr(self, name))


@dataclass(frozen=True, slots=True)
class OptimizerConfig:
    name: str = "adamw"
    lr: float = 3.0e-4
    betas: tuple[float, float] = (0.9, 0.95)
    eps: float = 1.0e-8
    weight_decay: float = 0.1
    clip_grad_norm: float | None = 1.0

    def __post_init__(self) -> None:
        if not isinstance(self.name, str):
            raise TypeError("optimizer.name must be a string")
        _set(self, "name", self.name.lower())
        _set(self, "betas", tuple(self.betas))
        if self.name != "adamw":
            raise ValueError("optimizer.name must be 'adamw' in the first implementation phase")
        _number("optimizer.lr", self.lr)
        _number("optimizer.eps", self.eps)
        _number("optimizer.weight_decay", self.weight_decay, allow_zero=True)
        if len(self.betas) != 2 or any(isinstance(b, bool) or not isinstance(b, (int, float))
                                       or not 0 <= b < 1 for b in self.betas):
            raise ValueError("optimizer.betas must contain two values in [0, 1)")
        if self.clip_grad_norm is not None:
            _number("optimizer.clip_grad_norm", self.clip_grad_norm)


@dataclass(frozen=True, slots=True)
class LearningRateSchedulerConfig:
    schedule: LearningRateSchedule = LearningRateSchedule.COSINE
    warmup_steps: int = 0
    decay_steps: int | None = None
    min_lr: float = 0.0

    def __post_init__(self) -> None:
        _set(self, "schedule", _enum("lr_scheduler.schedule", LearningRateSchedule, self.schedule))
        _int("lr_scheduler.warmup_steps", self.warmup_steps, minimum=0)
        if self.decay_steps is not None:
            _int("lr_scheduler.decay_steps", self.decay_steps)
        _number("lr_scheduler.min_lr", self.min_lr, allow_zero=True)


@dataclass(frozen=True, slots=True)
class TrainingConfig:
    micro_batch_size: int = 1
    gradient_accumulation_steps: int = 1
    max_steps: int = 1000
    seed: int = 1234
    log_interval: int = 10

    def __post_init__(self) -> None:
        for name in ("micro_batch_size", "gradient_accumulation_steps", "max_steps",
                     "log_interval"):
            _int(f"training.{name}", getattr(self, name))
        if isinstance(self.seed, bool) or not isinstance(self.seed, int) or self.seed < 0:
            raise ValueError("training.seed must be a non-negative integer")

    def global_batch_size(self, parallel: ParallelConfig, *, world_size: int | None = None) -> int:
        dp = parallel.resolve_data_parallel_size(world_size)
        return self.micro_batch_size * self.gradient_accumulation_steps * dp * parallel.expert


@dataclass(frozen=True, slots=True)
class CheckpointConfig:
    directory: Path = Path("checkpoints/gpt")
    save_interval: int = 500
    async_save: bool = False
    keep_last: int = 2
    save_final: bool = True
    save_best_validation: bool = True

    def __post_init__(self) -> None:
        _set(self, "directory", Path(self.directory))
        _int("checkpoint.save_interval", self.save_interval, minimum=0)
        _int("checkpoint.keep_last", self.keep_last)
        for name in ("async_save", "save_final", "save_best_validation"):
            _bool(f"checkpoint.{name}", getattr(self, name))


@dataclass(frozen=True, slots=True)
class TokenizerConfig:
    path: Path
    append_eos: bool = True

    def __post_init__(self) -> None:
        if not isinstance(self.path, (str, Path)):
            raise TypeError("data.tokenizer.path must be a filesystem path string")
        if isinstance(self.path, str) and not self.path.strip():
            raise ValueError("data.tokenizer.path must not be empty")
        _set(self, "path", Path(self.path))
        _bool("data.tokenizer.append_eos", self.append_eos)


@dataclass(frozen=True, slots=True)
class DataConfig:
    path: Path | None = None
    mmap_path: Path | None = None
    text_path: Path | None = None
    text_key: str = "text"
    tokenizer: TokenizerConfig | None = None
    num_workers: int = 0
    shuffle: bool = True
    packed_sequences: bool = False

    def __post_init__(self) -> None:
        for name in ("path", "mmap_path", "text_path"):
            _set(self, name, _path(f"data.{name}", getattr(self, name)))
        if not isinstance(self.text_key, str):
            raise TypeError("data.text_key must be a string")
        if not self.text_key.strip():
            raise ValueError("data.text_key must not be empty")
        if self.tokenizer is not None and not isinstance(self.tokenizer, TokenizerConfig):
            raise TypeError("data.tokenizer must be a TokenizerConfig or null")
        _int("data.num_workers", self.num_workers, minimum=0)
        _bool("data.shuffle", self.shuffle)
        _bool("data.packed_sequences", self.packed_sequences)


@dataclass(frozen=True, slots=True)
class ValidationConfig:
    interval: int = 0
    batches: int = 10
    data: DataConfig | None = None

    def __post_init__(self) -> None:
        _int("validation.interval", self.interval, minimum=0)
        _int("validation.batches", self.batches)
        if self.data is not None and not isinstance(self.data, DataConfig):
            raise TypeError("validation.data must be a DataConfig or null")


@dataclass(frozen=True, slots=True)
class WandbConfig:
    enabled: bool = False
    project: str = "nano-megatron"
    entity: str | None = None
    name: str | None = None
    group: str | None = None
    tags: tuple[str, ...] = ()
    mode: str = "online"
    directory: Path | None = None
    run_id: str | None = None

    def __post_init__(self) -> None:
        _bool("wandb.enabled", self.enabled)
        if not isinstance(self.project, str) or not self.project.strip():
            raise ValueError("wandb.project must be a non-empty string")
        _set(self, "project", self.project.strip())
        for name in ("entity", "name", "group", "run_id"):
            v = getattr(self, name)
            if v is not None and (not isinstance(v, str) or not v.strip()):
                raise ValueError(f"wandb.{name} must be a non-empty string or null")
            if isinstance(v, str):
                _set(self, name, v.strip())
        if isinstance(self.tags, str):
            raise TypeError("wandb.tags must be a sequence of strings, not a string")
        tags = tuple(self.tags)
        if any(not isinstance(t, str) or not t.strip() for t in tags):
            raise ValueError("wandb.tags must contain non-empty strings")
        _set(self, "tags", tuple(t.strip() for t in tags))
        if not isinstance(self.mode, str):
            raise TypeError("wandb.mode must be a string")
        mode = self.mode.strip().lower()
        if mode not in ("online", "offline", "disabled"):
            raise ValueError("wandb.mode must be online, offline, or disabled")
        _set(self, "mode", mode)
        _set(self, "directory", _path("wandb.directory", self.directory))


@dataclass(frozen=True, slots=True)
class TrainConfig:
    distributed: DistributedConfig = field(default_factory=DistributedConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    model: GPTConfig = field(default_factory=GPTConfig)
    precision: PrecisionConfig = field(default_factory=PrecisionConfig)
    kernels: KernelConfig = field(default_factory=KernelConfig)
    data_parallel: DataParallelConfig = field(default_factory=DataParallelConfig)
    pipeline: PipelineConfig = field(default_factory=PipelineConfig)
    context_parallel: ContextParallelConfig = field(default_factory=ContextParallelConfig)
    activation_checkpoint: ActivationCheckpointConfig = field(
        default_factory=ActivationCheckpointConfig)
    offload: OffloadConfig = field(default_factory=OffloadConfig)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    lr_scheduler: LearningRateSchedulerConfig = field(default_factory=LearningRateSchedulerConfig)
    training: TrainingConfig = field(default_factory=TrainingConfig)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    data: DataConfig = field(default_factory=DataConfig)
    validation: ValidationConfig = field(default_factory=ValidationConfig)
    wandb: WandbConfig = field(default_factory=WandbConfig)

    def global_batch_size(self, *, world_size: int | None = None) -> int:
        return self.training.global_batch_size(self.parallel, world_size=world_size)
