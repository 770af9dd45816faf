"""Cross-block configuration rules.

Same rule set as the reference (src/nano_megatron/config/validation.py:60-298):
divisibility of H/F/heads/kv_heads by TP and of S by CP, SP needs (S/CP) % TP
== 0, layers >= PP*v, interleaved-schedule constraints, precision/mode and
offload/mode compatibility, CP needs dropout 0, packed sequences rejected, data
source exclusivity, LR-schedule horizon checks. Errors are collected and
raised together; notices come back as warnings.
"""

from __future__ import annotations

from dataclasses import dataclass

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


def _data_source_rules(data: DataConfig, prefix: str, require: bool) -> list[str]:
    errors = []
    n = sum(x is not None for x in (data.path, data.mmap_path, data.text_path))
    if n > 1:
        errors.append(f"{prefix}.path, {prefix}.mmap_path, and {prefix}.text_path are mutually "
                      "exclusive; at most one may be set")
    if require and n == 0:
        errors.append(f"{prefix} must configure path, mmap_path, or text_path")
    if data.text_path is not None and data.tokenizer is None:
        errors.append(f"{prefix}.text_path requires {prefix}.tokenizer")
    if data.tokenizer is not None and n == 0:
        errors.append(f"{prefix}.tokenizer requires {prefix}.path, {prefix}.mmap_path, or "
                      f"{prefix}.text_path")
    if data.packed_sequences:
        errors.append(f"{prefix}.packed_sequences=true is not supported; document-aware "
                      "attention masks are not implemented")
    return errors


def validate_config(config: TrainConfig, *, world_size: int | None = None) -> ValidationResult:
    errors: list[str] = []
    notes: list[str] = []
    par, model, train = config.parallel, config.model, config.training

    horizon = train.max_steps if config.lr_scheduler.decay_steps is None \
        else config.lr_scheduler.decay_steps
    if config.lr_scheduler.warmup_steps > horizon:
        errors.append("lr_scheduler.warmup_steps cannot exceed the effective decay horizon: "
                      f"{config.lr_scheduler.warmup_steps} > {horizon}")
    if config.lr_scheduler.min_lr > config.optimizer.lr:
        errors.append(f"lr_scheduler.min_lr cannot exceed optimizer.lr: "
                      f"{config.lr_scheduler.min_lr} > {config.optimizer.lr}")
    if (config.precision.compute is PrecisionDType.FLOAT32
            and config.precision.params is not PrecisionDType.FLOAT32):
        errors.append("precision.compute=float32 requires precision.params=float32; "
                      "low-precision parameters cannot guarantee FP32 compute")

    dp = None
    try:
        if world_size is not None or par.data is not None:
            dp = par.resolve_data_parallel_size(world_size)
    except (TypeError, ValueError) as error:
        errors.append(str(error))

    for value, div, vname, dname in (
        (model.hidden_size, par.tensor, "model.hidden_size", "parallel.tensor"),
        (model.ffn_hidden_size, par.tensor, "model.ffn_hidden_size", "parallel.tensor"),
        (model.heads, par.tensor, "model.heads", "parallel.tensor"),
        (model.num_kv_heads, par.tensor, "model.kv_heads", "parallel.tensor"),
        (model.seq_length, par.context, "model.seq_length", "parallel.context"),
    ):
        if value % div:
            errors.append(f"{vname} ({value}) must be divisible by {dname} ({div})")
    if config.context_parallel.load_balance and model.seq_length % (2 * par.context):
        errors.append("context_parallel.load_balance requires model.seq_length divisible by "
                      f"2 * parallel.context ({2 * par.context})")

    if par.sequence_parallel:
        local = model.seq_length // par.context
        if model.seq_length % par.context == 0 and local % par.tensor:
            errors.append("sequence parallelism requires (model.seq_length / parallel.context) "
                          f"to be divisible by parallel.tensor; got {local} and {par.tensor}")
        if par.tensor == 1:
            notes.append("parallel.sequence_parallel is enabled with TP=1 and therefore has no "
                         "sharding effect")

    v = config.pipeline.virtual_stages_per_rank
    stages = par.pipeline * v
    if model.layers < stages:
        errors.append(f"model.layers ({model.layers}) must be >= parallel.pipeline * "
                      f"pipeline.virtual_stages_per_rank ({par.pipeline} * {v} = {stages})")
    gas = train.gradient_accumulation_steps
    if config.pipeline.schedule is PipelineSchedule.INTERLEAVED_ONE_F_ONE_B:
        if par.pipeline == 1:
            errors.append("interleaved_1f1b requires parallel.pipeline > 1")
        if v < 2:
            errors.append("interleaved_1f1b requires pipeline.virtual_stages_per_rank >= 2")
        if gas < par.pipeline:
            errors.append("interleaved_1f1b requires gradient_accumulation_steps >= "
                          "parallel.pipeline")
        if gas % par.pipeline:
            errors.append("interleaved_1f1b requires gradient_accumulation_steps to be "
                          "divisible by parallel.pipeline")
        if model.layers % stages:
            notes.append("interleaved pipeline chunks have uneven layer counts because "
                         "model.layers is not divisible by PP * virtual_stages_per_rank")
    elif v != 1:
        errors.append("pipeline.virtual_stages_per_rank > 1 requires schedule=interleaved_1f1b")
    if config.pipeline.schedule is PipelineSchedule.ONE_F_ONE_B and gas < par.pipeline:
        notes.append(f"1F1B pipeline utilization is low when gradient_accumulation_steps ({gas}) "
                     f"< PP ({par.pipeline})")

    errors += _data_source_rules(config.data, "data", False)
    vdata = config.validation.data
    if config.validation.interval > 0:
        if vdata is None:
            errors.append("validation.interval > 0 requires validation.data")
        else:
            errors += _data_source_rules(vdata, "validation.data", True)
    elif vdata is not None:
        notes.append("validation.data is configured but validation.interval=0 disables it")
    if (vdata is not None and vdata.tokenizer is not None and config.data.tokenizer is not None
            and vdata.tokenizer.path != config.data.tokenizer.path):
        errors.append("training and validation data must use the same tokenizer artifact")
    if par.context > 1 and model.dropout > 0.0:
        errors.append("model.dropout must be 0 when context parallelism is enabled in phase one; "
                      "CP attention dropout is not implemented")

    mode = config.data_parallel.mode
    if config.precision.params is PrecisionDType.FLOAT16 and mode in (DataParallelMode.DDP,
                                                                      DataParallelMode.ZERO3):
        errors.append(f"precision.params=float16 is not supported with data_parallel.mode="
                      f"{mode.value}; DDP and ZeRO-3 do not maintain FP32 master parameters. Use "
                      "precision.params=float32 with precision.compute=float16, or use "
                      "ZeRO-1/ZeRO-2 with their FP32 master shards")
    off = config.offload
    if off.optimizer_state:
        if mode is DataParallelMode.DDP:
            errors.append("optimizer-state offload requires data_parallel.mode zero1 or zero2")
        elif mode is DataParallelMode.ZERO3:
            errors.append("optimizer_state offload is not a separate ZeRO-3 option; use "
                          "offload.zero3_params_and_grads with the FSDP2 CPU offload policy")
    if off.zero3_params_and_grads and mode is not DataParallelMode.ZERO3:
        errors.append("offload.zero3_params_and_grads requires data_parallel.mode=zero3")
    if config.data_parallel.overlap_grad_reduce and mode is DataParallelMode.ZERO3:
        notes.append("data_parallel.overlap_grad_reduce is managed internally in zero3 mode")
    elif (config.data_parallel.overlap_grad_reduce and dp is not None
          and dp * par.expert * par.context == 1):
        notes.append("data_parallel.overlap_grad_reduce has no communication effect on a "
                     "size-one replica group")
    if config.pipeline.overlap_p2p and par.pipeline == 1:
        notes.append("pipeline.overlap_p2p has no communication effect when parallel.pipeline=1")
    if config.pipeline.dynamic_activation_shapes and par.pipeline == 1:
        notes.append("pipeline.dynamic_activation_shapes has no communication effect when "
                     "parallel.pipeline=1")
    ac = config.activation_checkpoint
    if ac.mode is ActivationCheckpointMode.SELECTIVE and not ac.selective_ops:
        errors.append("selective activation checkpointing requires at least one selective op")
    if ac.mode is ActivationCheckpointMode.NONE and ac.offload_saved_tensors:
        errors.append("activation_checkpoint.offload_saved_tensors requires activation "
                      "checkpointing to be enabled")
    if par.expert > 1:
        notes.append("dense GPT with EP>1 treats EP ranks as additional dense batch replicas; "
                     "MoE token dispatch is not implemented in phase one")
    dense = None if dp is None else dp * par.expert * par.context
    if mode is DataParallelMode.ZERO3 and dense == 1:
        notes.append("ZeRO-3 replica mesh has size 1 and will degenerate to local execution")
        if off.zero3_params_and_grads:
            errors.append("offload.zero3_params_and_grads requires an active ZeRO-3 replica "
                          "mesh; the configured mesh has size 1")
    if errors:
        raise ConfigValidationError("invalid Nano-Megatron configuration:\n- "
                                    + "\n- ".join(errors))
    gbs = None if dp is None else train.micro_batch_size * gas * dp * par.expert
    return ValidationResult(world_size, dp, model.padded_vocab_size(par.tensor), gbs, tuple(notes))


validate_train_config = validate_config
