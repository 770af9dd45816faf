"""Cross-block configuration rules.

Each block validates its own fields on construction (:mod:`.schema`); the rules here look
at combinations of blocks. They accept, reject and warn on the same configurations as the
reference's validator (src/nano_megatron/config/validation.py:60-298); the wording of the
messages is this project's.

Design: every rule is a small function registered with :func:`_rule` and evaluated in
registration order against one :class:`_Facts` object (the config plus the data-parallel
size resolved once). A rule reports problems with ``facts.fail(...)`` and notices with
``facts.note(...)``. All failures are collected and raised together as one
:class:`ConfigValidationError`; notices come back in :class:`ValidationResult`.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field

from .schema import (
    ActivationCheckpointMode,
    DataConfig,
    DataParallelMode,
    PipelineSchedule,
    PrecisionDType,
    TrainConfig,
)


class ConfigValidationError(ValueError):
    """Individually valid blocks that cannot be combined."""


@dataclass(frozen=True, slots=True)
class ValidationResult:
    world_size: int | None
    data_parallel_size: int | None
    padded_vocab_size: int
    global_batch_size: int | None
    warnings: tuple[str, ...] = ()


@dataclass
class _Facts:
    config: TrainConfig
    world_size: int | None
    dp: int | None = None               # resolved data-parallel size, when known
    failures: list[str] = field(default_factory=list)
    notices: list[str] = field(default_factory=list)

    def fail(self, text: str) -> None:
        self.failures.append(text)

    def note(self, text: str) -> None:
        self.notices.append(text)

    @property
    def replicas(self) -> int | None:
        """Dense replicas of one model shard: DP x EP x CP (None until DP is known)."""
        par = self.config.parallel
        return None if self.dp is None else self.dp * par.expert * par.context


_RULES: list[Callable[[_Facts], None]] = []


def _rule(fn: Callable[[_Facts], None]) -> Callable[[_Facts], None]:
    _RULES.append(fn)
    return fn


# ---------------------------------------------------------------- optimizer schedule
@_rule
def _schedule_horizon(f: _Facts) -> None:
    sched, opt = f.config.lr_scheduler, f.config.optimizer
    horizon = sched.decay_steps if sched.decay_steps is not None else f.config.training.max_steps
    if sched.warmup_steps > horizon:
        f.fail(f"warm-up of {sched.warmup_steps} steps (lr_scheduler.warmup_steps) is longer "
               f"than the {horizon}-step decay horizon")
    if sched.min_lr > opt.lr:
        f.fail(f"lr_scheduler.min_lr={sched.min_lr} is above the peak optimizer.lr={opt.lr}")


@_rule
def _precision_pair(f: _Facts) -> None:
    prec = f.config.precision
    if prec.compute is PrecisionDType.FLOAT32 and prec.params is not PrecisionDType.FLOAT32:
        f.fail("fp32 compute (precision.compute=float32) needs fp32 parameters "
               f"(precision.params is {prec.params.value})")


# ---------------------------------------------------------------- topology
@_rule
def _resolve_topology(f: _Facts) -> None:
    par = f.config.parallel
    if f.world_size is None and par.data is None:
        return
    try:
        f.dp = par.resolve_data_parallel_size(f.world_size)
    except (TypeError, ValueError) as error:
        f.fail(str(error))


@_rule
def _shard_divisibility(f: _Facts) -> None:
    par, model = f.config.parallel, f.config.model
    checks = (("model.hidden_size", model.hidden_size, "parallel.tensor", par.tensor),
              ("model.ffn_hidden_size", model.ffn_hidden_size, "parallel.tensor", par.tensor),
              ("model.heads", model.heads, "parallel.tensor", par.tensor),
              ("model.kv_heads", model.num_kv_heads, "parallel.tensor", par.tensor),
              ("model.seq_length", model.seq_length, "parallel.context", par.context))
    for what, value, by, size in checks:
        if value % size:
            f.fail(f"{what}={value} cannot be split evenly over {by}={size}")
    if f.config.context_parallel.load_balance and model.seq_length % (2 * par.context):
        f.fail(f"zig-zag chunks (context_parallel.load_balance) need model.seq_length="
               f"{model.seq_length} to be a multiple of 2 x parallel.context = {2 * par.context}")


@_rule
def _sequence_parallel(f: _Facts) -> None:
    par, seq = f.config.parallel, f.config.model.seq_length
    if not par.sequence_parallel:
        return
    per_cp_rank = seq // par.context
    if seq % par.context == 0 and per_cp_rank % par.tensor:
        f.fail(f"sequence parallelism splits each context-parallel shard ({per_cp_rank} tokens) "
               f"over parallel.tensor={par.tensor}, which does not divide it")
    if par.tensor == 1:
        f.note("parallel.sequence_parallel does nothing without tensor parallelism (TP=1)")


# ---------------------------------------------------------------- pipeline
@_rule
def _pipeline_shape(f: _Facts) -> None:
    cfg = f.config
    pp, virt = cfg.parallel.pipeline, cfg.pipeline.virtual_stages_per_rank
    chunks = pp * virt
    layers, gas = cfg.model.layers, cfg.training.gradient_accumulation_steps
    if layers < chunks:
        f.fail(f"{layers} layers cannot fill {chunks} pipeline chunks "
               f"(parallel.pipeline={pp} x pipeline.virtual_stages_per_rank={virt})")
    schedule = cfg.pipeline.schedule
    if schedule is PipelineSchedule.INTERLEAVED_ONE_F_ONE_B:
        if pp == 1:
            f.fail("the interleaved_1f1b schedule needs parallel.pipeline > 1")
        if virt < 2:
            f.fail("the interleaved_1f1b schedule needs at least 2 virtual stages per rank")
        if gas < pp:
            f.fail(f"the interleaved_1f1b schedule needs at least parallel.pipeline={pp} "
                   f"microbatches per step (training.gradient_accumulation_steps={gas})")
        if gas % pp:
            f.fail(f"the interleaved_1f1b schedule needs the microbatch count ({gas}) to be a "
                   f"multiple of parallel.pipeline={pp}")
        if layers % chunks:
            f.note(f"{layers} layers over {chunks} interleaved chunks: chunks get unequal "
                   "layer counts")
    elif virt != 1:
        f.fail("pipeline.virtual_stages_per_rank other than 1 is only meaningful with the "
               "interleaved_1f1b schedule")
    if schedule is PipelineSchedule.ONE_F_ONE_B and gas < pp:
        f.note(f"1F1B with fewer microbatches ({gas}) than pipeline stages ({pp}) leaves "
               "stages idle")
    if cfg.pipeline.overlap_p2p and pp == 1:
        f.note("pipeline.overlap_p2p has no effect on a single pipeline stage")
    if cfg.pipeline.dynamic_activation_shapes and pp == 1:
        f.note("pipeline.dynamic_activation_shapes has no effect on a single pipeline stage")


# ---------------------------------------------------------------- data
def _data_block(f: _Facts, data: DataConfig, where: str, required: bool) -> None:
    sources = [name for name in ("path", "mmap_path", "text_path")
               if getattr(data, name) is not None]
    if len(sources) > 1:
        f.fail(f"{where}: choose one data source, not {' and '.join(sources)}")
    if required and not sources:
        f.fail(f"{where}: a data source (path, mmap_path or text_path) is required")
    if data.text_path is not None and data.tokenizer is None:
        f.fail(f"{where}: raw text (text_path) needs a tokenizer")
    if data.tokenizer is not None and not sources:
        f.fail(f"{where}: a tokenizer is set but no data source is")
    if data.packed_sequences:
        f.fail(f"{where}: packed_sequences needs document-aware attention masks, which are "
               "not supported")


@_rule
def _data_sources(f: _Facts) -> None:
    cfg = f.config
    _data_block(f, cfg.data, "data", required=False)
    val = cfg.validation.data
    if cfg.validation.interval > 0:
        if val is None:
            f.fail("periodic validation (validation.interval > 0) needs validation.data")
        else:
            _data_block(f, val, "validation.data", required=True)
    elif val is not None:
        f.note("validation.data is set but validation.interval=0, so it is never used")
    if (val is not None and val.tokenizer is not None and cfg.data.tokenizer is not None
            and val.tokenizer.path != cfg.data.tokenizer.path):
        f.fail("training and validation data name different tokenizer artifacts")


@_rule
def _context_parallel_dropout(f: _Facts) -> None:
    if f.config.parallel.context > 1 and f.config.model.dropout > 0.0:
        f.fail("attention dropout is not available under context parallelism; set "
               "model.dropout to 0")


# ---------------------------------------------------------------- data parallel, offload
@_rule
def _data_parallel_modes(f: _Facts) -> None:
    cfg = f.config
    mode, off = cfg.data_parallel.mode, cfg.offload
    if cfg.precision.params is PrecisionDType.FLOAT16 and mode in (DataParallelMode.DDP,
                                                                   DataParallelMode.ZERO3):
        f.fail(f"fp16 parameters need fp32 master copies, which data_parallel.mode="
               f"{mode.value} does not keep; use fp32 parameters with fp16 compute, or "
               "ZeRO-1/2")
    if off.optimizer_state and mode is DataParallelMode.DDP:
        f.fail("offload.optimizer_state works on sharded optimizer state: use "
               "data_parallel.mode zero1 or zero2")
    elif off.optimizer_state and mode is DataParallelMode.ZERO3:
        f.fail("under ZeRO-3 optimizer state moves with offload.zero3_params_and_grads, not "
               "offload.optimizer_state")
    if off.zero3_params_and_grads and mode is not DataParallelMode.ZERO3:
        f.fail(f"offload.zero3_params_and_grads applies to data_parallel.mode=zero3 only "
               f"(got {mode.value})")
    if cfg.data_parallel.overlap_grad_reduce:
        if mode is DataParallelMode.ZERO3:
            f.note("ZeRO-3 schedules its own gradient reduction; "
                   "data_parallel.overlap_grad_reduce is ignored")
        elif f.dp is not None and f.replicas == 1:
            f.note("data_parallel.overlap_grad_reduce has nothing to overlap with a single "
                   "replica")
    if mode is DataParallelMode.ZERO3 and f.replicas == 1:
        f.note("ZeRO-3 over a single replica shards nothing and runs locally")
        if off.zero3_params_and_grads:
            f.fail("offload.zero3_params_and_grads needs more than one ZeRO-3 replica")


@_rule
def _activation_checkpointing(f: _Facts) -> None:
    ac = f.config.activation_checkpoint
    if ac.mode is ActivationCheckpointMode.SELECTIVE and not ac.selective_ops:
        f.fail("selective activation checkpointing has no ops to recompute")
    if ac.mode is ActivationCheckpointMode.NONE and ac.offload_saved_tensors:
        f.fail("activation_checkpoint.offload_saved_tensors needs a checkpointing mode "
               "(full or selective)")


@_rule
def _expert_parallel(f: _Facts) -> None:
    if f.config.parallel.expert > 1:
        f.note("the dense GPT has no experts: expert-parallel ranks act as extra data-parallel "
               "replicas")


def validate_config(config: TrainConfig, *, world_size: int | None = None) -> ValidationResult:
    facts = _Facts(config, world_size)
    for rule in _RULES:
        rule(facts)
    if facts.failures:
        raise ConfigValidationError("configuration rejected:\n  * "
                                    + "\n  * ".join(facts.failures))
    par, train = config.parallel, config.training
    batch = (None if facts.dp is None else
             train.micro_batch_size * train.gradient_accumulation_steps * facts.dp * par.expert)
    return ValidationResult(world_size, facts.dp, config.model.padded_vocab_size(par.tensor),
                            batch, tuple(facts.notices))


validate_train_config = validate_config
