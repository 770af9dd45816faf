"""Typed configuration blocks.

The YAML schema is the reference's (src/nano_megatron/config/schema.py:60-665): the same
17 blocks, field names and defaults, and the same accept/reject decisions, so reference
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

How blocks validate themselves: every block is a frozen dataclass deriving from
:class:`_Block`. A field's constraints travel with the field as metadata (:func:`_spec`);
after construction one generic checker walks the fields and, guided by each field's type
hint, rejects or normalises the value: booleans must be real booleans; integers real
integers at or above their lower bound (1 unless the spec says otherwise); numbers real
numbers within their bounds; enums are coerced from their string values; paths from
strings; text is stripped and/or lower-cased where the spec asks. Wrong types raise
``TypeError`` and out-of-range values ``ValueError``, each naming the dotted field. What
involves more than one field, or a field the generic rules cannot express, is checked in
the block's ``_cross_check``.
"""

from __future__ import annotations

import dataclasses
import types
import typing
from dataclasses import dataclass, field
from enum import StrEnum
from pathlib import Path

from nano_megatron_b200.parallel.axes import DEFAULT_RANK_ORDER, ParallelAxis, normalize_rank_order


# ------------------------------------------------------------------ field specs
@dataclass(frozen=True, slots=True)
class _Spec:
    low: float | None = None     # lower bound (inclusive, or exclusive with `above`)
    above: bool = False
    below: float | None = None   # exclusive upper bound for numbers
    strip: bool = False          # text: strip surrounding whitespace
    lower: bool = False          # text: lower-case
    nonblank: bool = False       # text / path: must contain a non-space character
    own: bool = False            # checked only by the block's _cross_check


_PLAIN = _Spec()


def _spec(default=dataclasses.MISSING, *, factory=dataclasses.MISSING, **rules):
    meta = {"spec": _Spec(**rules)}
    if factory is not dataclasses.MISSING:
        return field(default_factory=factory, metadata=meta)
    return field(default=default, metadata=meta)


_HINT_CACHE: dict[type, dict[str, object]] = {}


def _field_hints(cls: type) -> dict[str, object]:
    hints = _HINT_CACHE.get(cls)
    if hints is None:
        hints = _HINT_CACHE[cls] = typing.get_type_hints(cls)
    return hints


def _checked(name: str, value, hint, spec: _Spec):
    """Validate one field value against its type hint and spec; return the stored value."""
    if typing.get_origin(hint) in (typing.Union, types.UnionType):
        if value is None:
            return None
        (hint,) = [arm for arm in typing.get_args(hint) if arm is not type(None)]
    if hint is bool:
        if not isinstance(value, bool):
            raise TypeError(f"{name}: expected true or false, found {value!r}")
        return value
    if hint is int or hint is float:
        kinds = (int,) if hint is int else (int, float)
        if isinstance(value, bool) or not isinstance(value, kinds):
            what = "a whole number" if hint is int else "a number"
            raise TypeError(f"{name}: expected {what}, found {value!r}")
        low = 1 if hint is int and spec.low is None else spec.low
        if low is not None and (value <= low if spec.above else value < low):
            raise ValueError(f"{name}: {value} is not {'above' if spec.above else 'at least'} "
                             f"{low}")
        if spec.below is not None and value >= spec.below:
            raise ValueError(f"{name}: {value} is not below {spec.below}")
        return value
    if isinstance(hint, type) and issubclass(hint, StrEnum):
        try:
            return hint(value)
        except (TypeError, ValueError) as error:
            allowed = " | ".join(member.value for member in hint)
            raise ValueError(f"{name}: {value!r} is not one of {allowed}") from error
    if hint is str:
        if not isinstance(value, str):
            raise TypeError(f"{name}: expected text, found {value!r}")
        if spec.nonblank and not value.strip():
            raise ValueError(f"{name}: must not be blank")
        text = value.strip() if spec.strip else value
        return text.lower() if spec.lower else text
    if hint is Path:
        if not isinstance(value, (str, Path)):
            raise TypeError(f"{name}: expected a filesystem path, found {value!r}")
        if spec.nonblank and isinstance(value, str) and not value.strip():
            raise ValueError(f"{name}: must not be blank")
        return Path(value)
    if dataclasses.is_dataclass(hint):
        if not isinstance(value, hint):
            raise TypeError(f"{name}: expected a {hint.__name__} block, found "
                            f"{type(value).__name__}")
        return value
    raise TypeError(f"{name}: no generic rule for type {hint!r}; give it an own check")


class _Block:
    __slots__ = ()
    SECTION = ""

    def __post_init__(self) -> None:
        hints = _field_hints(type(self))
        for f in dataclasses.fields(self):
            spec = f.metadata.get("spec", _PLAIN)
            if spec.own:
                continue
            value = getattr(self, f.name)
            stored = _checked(f"{self.SECTION}.{f.name}", value, hints[f.name], spec)
            if stored is not value:
                object.__setattr__(self, f.name, stored)
        self._cross_check()

    def _cross_check(self) -> None:
        """Rules over several fields, and fields marked ``own``."""

    def _store(self, name: str, value) -> None:
        object.__setattr__(self, name, value)


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
class DistributedConfig(_Block):
    SECTION = "distributed"
    backend: str = _spec("auto", nonblank=True, strip=True, lower=True)
    timeout_minutes: int = 30
    device: str = _spec("auto", nonblank=True, strip=True, lower=True)
    init_method: str = _spec("env://", nonblank=True, strip=True)


@dataclass(frozen=True, slots=True)
class ParallelConfig(_Block):
    SECTION = "parallel"
    tensor: int = 1
    pipeline: int = 1
    context: int = 1
    expert: int = 1
    data: int | None = None
    order: tuple[ParallelAxis, ...] = _spec(DEFAULT_RANK_ORDER, own=True)
    sequence_parallel: bool = False

    def _cross_check(self) -> None:
        self._store("order", normalize_rank_order(self.order))

    @property
    def tensor_parallel_size(self) -> int:
        return self.tensor

    @property
    def pipeline_parallel_size(self) -> int:
        return self.pipeline

    @property
    def context_parallel_size(self) -> int:
        return self.context

    @property
    def expert_parallel_size(self) -> int:
        return self.expert

    @property
    def data_parallel_size(self) -> int:
        if self.data is None:
            raise ValueError("parallel.data is still null: resolve it against a world size "
                             "first")
        return self.data

    @property
    def model_parallel_size(self) -> int:
        return self.tensor * self.pipeline * self.context * self.expert

    @property
    def configured_world_size(self) -> int | None:
        return None if self.data is None else self.model_parallel_size * self.data

    def resolve_data_parallel_size(self, world_size: int | None) -> int:
        """DP size implied by ``world_size`` (or the configured one, checked against it)."""
        if world_size is not None:
            _checked("world_size", world_size, int, _PLAIN)
        shard = self.model_parallel_size
        layout = (f"TP {self.tensor} x PP {self.pipeline} x CP {self.context} x "
                  f"EP {self.expert}")
        if self.data is None:
            if world_size is None:
                raise ValueError("parallel.data is null, so a world size is needed to derive it")
            if world_size % shard:
                raise ValueError(f"{world_size} ranks cannot be split into model replicas of "
                                 f"{layout} = {shard} ranks")
            return world_size // shard
        if world_size is not None and shard * self.data != world_size:
            raise ValueError(f"{layout} x DP {self.data} = {shard * self.data} ranks, but the "
                             f"world has {world_size}")
        return self.data

    def resolved(self, world_size: int) -> "ParallelConfig":
        return dataclasses.replace(self, data=self.resolve_data_parallel_size(world_size))


@dataclass(frozen=True, slots=True)
class GPTConfig(_Block):
    SECTION = "model"
    layers: int = 12
    hidden_size: int = 768
    ffn_hidden_size: int = 2048
    heads: int = 12
    kv_heads: int | None = None
    seq_length: int = 2048
    vocab_size: int = 50304
    rope_theta: float = _spec(10000.0, low=0, above=True)
    dropout: float = _spec(0.0, low=0, below=1)
    tie_embeddings: bool = True
    norm_epsilon: float = _spec(1.0e-5, low=0, above=True)
    bias: bool = False

    def _cross_check(self) -> None:
        if self.hidden_size % self.heads:
            raise ValueError(f"model: hidden_size {self.hidden_size} does not split into "
                             f"{self.heads} equal heads")
        kv = self.num_kv_heads
        if kv > self.heads or self.heads % kv:
            raise ValueError(f"model: {self.heads} query heads cannot share {kv} key/value "
                             "heads evenly (kv_heads must divide heads)")

    @property
    def num_layers(self) -> int:
        return self.layers

    @property
    def num_attention_heads(self) -> int:
        return self.heads

    @property
    def num_kv_heads(self) -> int:
        return self.heads if self.kv_heads is None else self.kv_heads

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.heads

    def padded_vocab_size(self, tensor_parallel_size: int) -> int:
        """Vocabulary rounded up to a multiple of the TP size (equal vocabulary shards)."""
        tp = _checked("tensor_parallel_size", tensor_parallel_size, int, _PLAIN)
        return (self.vocab_size + tp - 1) // tp * tp


@dataclass(frozen=True, slots=True)
class PrecisionConfig(_Block):
    SECTION = "precision"
    params: PrecisionDType = PrecisionDType.BFLOAT16
    compute: PrecisionDType = PrecisionDType.BFLOAT16
    grad_reduce: PrecisionDType = PrecisionDType.FLOAT32


@dataclass(frozen=True, slots=True)
class KernelConfig(_Block):
    SECTION = "kernels"
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


@dataclass(frozen=True, slots=True)
class DataParallelConfig(_Block):
    SECTION = "data_parallel"
    mode: DataParallelMode = DataParallelMode.DDP
    bucket_bytes: int = 256 * 1024 * 1024
    overlap_grad_reduce: bool = False
    reshard_after_forward: bool = True


@dataclass(frozen=True, slots=True)
class PipelineConfig(_Block):
    SECTION = "pipeline"
    schedule: PipelineSchedule = PipelineSchedule.ONE_F_ONE_B
    activation_dtype: PrecisionDType | None = None
    overlap_p2p: bool = False
    virtual_stages_per_rank: int = 1
    dynamic_activation_shapes: bool = False


@dataclass(frozen=True, slots=True)
class ContextParallelConfig(_Block):
    SECTION = "context_parallel"
    backend: ContextParallelBackend = ContextParallelBackend.ALL_GATHER
    dropout: float = _spec(0.0, own=True)
    load_balance: bool = False

    def _cross_check(self) -> None:
        d = _checked("context_parallel.dropout", self.dropout, float, _PLAIN)
        if d != 0.0:
            raise ValueError("context_parallel.dropout: attention dropout is not implemented "
                             "for context parallelism; only 0 is accepted")


_CHECKPOINTABLE_OPS = ("attention", "mlp")


@dataclass(frozen=True, slots=True)
class ActivationCheckpointConfig(_Block):
    SECTION = "activation_checkpoint"
    mode: ActivationCheckpointMode = ActivationCheckpointMode.NONE
    block_interval: int = 1
    selective_ops: tuple[str, ...] = _spec(_CHECKPOINTABLE_OPS, own=True)
    use_reentrant: bool = False
    offload_saved_tensors: bool = False

    def _cross_check(self) -> None:
        ops = tuple(self.selective_ops)
        self._store("selective_ops", ops)
        if not ops:
            raise ValueError("activation_checkpoint.selective_ops: name at least one op")
        extra = sorted(set(ops) - set(_CHECKPOINTABLE_OPS))
        if extra:
            raise ValueError(f"activation_checkpoint.selective_ops: {', '.join(extra)} cannot "
                             f"be recomputed (choose from {', '.join(_CHECKPOINTABLE_OPS)})")
        if self.use_reentrant:
            raise ValueError("activation_checkpoint.use_reentrant: only non-reentrant "
                             "checkpointing is implemented")


@dataclass(frozen=True, slots=True)
class OffloadConfig(_Block):
    SECTION = "offload"
    optimizer_state: bool = False
    zero3_params_and_grads: bool = False
    activations: bool = False
    pin_memory: bool = True
    non_blocking: bool = True


@dataclass(frozen=True, slots=True)
class OptimizerConfig(_Block):
    SECTION = "optimizer"
    name: str = _spec("adamw", lower=True)
    lr: float = _spec(3.0e-4, low=0, above=True)
    betas: tuple[float, float] = _spec((0.9, 0.95), own=True)
    eps: float = _spec(1.0e-8, low=0, above=True)
    weight_decay: float = _spec(0.1, low=0)
    clip_grad_norm: float | None = _spec(1.0, low=0, above=True)

    def _cross_check(self) -> None:
        betas = tuple(self.betas)
        self._store("betas", betas)
        if self.name != "adamw":
            raise ValueError(f"optimizer.name: {self.name!r} is not available (only adamw)")
        in_range = [not isinstance(b, bool) and isinstance(b, (int, float)) and 0 <= b < 1
                    for b in betas]
        if len(betas) != 2 or not all(in_range):
            raise ValueError(f"optimizer.betas: need two coefficients in [0, 1), got {betas!r}")


@dataclass(frozen=True, slots=True)
class LearningRateSchedulerConfig(_Block):
    SECTION = "lr_scheduler"
    schedule: LearningRateSchedule = LearningRateSchedule.COSINE
    warmup_steps: int = _spec(0, low=0)
    decay_steps: int | None = None
    min_lr: float = _spec(0.0, low=0)


@dataclass(frozen=True, slots=True)
class TrainingConfig(_Block):
    SECTION = "training"
    micro_batch_size: int = 1
    gradient_accumulation_steps: int = 1
    max_steps: int = 1000
    seed: int = _spec(1234, low=0)
    log_interval: int = 10

    def global_batch_size(self, parallel: ParallelConfig, *, world_size: int | None = None) -> int:
        """Sequences per optimizer step over every replica (DP x EP)."""
        dp = parallel.resolve_data_parallel_size(world_size)
        return self.micro_batch_size * self.gradient_accumulation_steps * dp * parallel.expert


@dataclass(frozen=True, slots=True)
class CheckpointConfig(_Block):
    SECTION = "checkpoint"
    directory: Path = Path("checkpoints/gpt")
    save_interval: int = _spec(500, low=0)
    async_save: bool = False
    keep_last: int = 2
    save_final: bool = True
    save_best_validation: bool = True


@dataclass(frozen=True, slots=True)
class TokenizerConfig(_Block):
    SECTION = "data.tokenizer"
    path: Path = _spec(nonblank=True)
    append_eos: bool = True


@dataclass(frozen=True, slots=True)
class DataConfig(_Block):
    SECTION = "data"
    path: Path | None = _spec(None, nonblank=True)
    mmap_path: Path | None = _spec(None, nonblank=True)
    text_path: Path | None = _spec(None, nonblank=True)
    text_key: str = _spec("text", nonblank=True)
    tokenizer: TokenizerConfig | None = None
    num_workers: int = _spec(0, low=0)
    shuffle: bool = True
    packed_sequences: bool = False


@dataclass(frozen=True, slots=True)
class ValidationConfig(_Block):
    SECTION = "validation"
    interval: int = _spec(0, low=0)
    batches: int = 10
    data: DataConfig | None = None


_WANDB_MODES = ("online", "offline", "disabled")


@dataclass(frozen=True, slots=True)
class WandbConfig(_Block):
    SECTION = "wandb"
    enabled: bool = False
    project: str = _spec("nano-megatron", nonblank=True, strip=True)
    entity: str | None = _spec(None, nonblank=True, strip=True)
    name: str | None = _spec(None, nonblank=True, strip=True)
    group: str | None = _spec(None, nonblank=True, strip=True)
    tags: tuple[str, ...] = _spec((), own=True)
    mode: str = _spec("online", strip=True, lower=True)
    directory: Path | None = _spec(None, nonblank=True)
    run_id: str | None = _spec(None, nonblank=True, strip=True)

    def _cross_check(self) -> None:
        if isinstance(self.tags, str):
            raise TypeError("wandb.tags: expected a list of tags, found a single string")
        tags = tuple(self.tags)
        if not all(isinstance(t, str) and t.strip() for t in tags):
            raise ValueError(f"wandb.tags: every tag must be non-blank text, got {tags!r}")
        self._store("tags", tuple(t.strip() for t in tags))
        if self.mode not in _WANDB_MODES:
            raise ValueError(f"wandb.mode: {self.mode!r} is not one of {' | '.join(_WANDB_MODES)}")


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
