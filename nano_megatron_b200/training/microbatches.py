"""Microbatch splitting of nested batches (reference: src/nano_megatron/training/microbatches.py)."""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import is_dataclass, replace
from typing import Any

import torch


def global_batch_size(micro_batch_size: int, gradient_accumulation_steps: int,
                      data_parallel_size: int, expert_parallel_size: int) -> int:
    vals = (micro_batch_size, gradient_accumulation_steps, data_parallel_size,
            expert_parallel_size)
    if any(v < 1 for v in vals):
        raise ValueError("batch and parallel sizes must be positive")
    return micro_batch_size * gradient_accumulation_steps * data_parallel_size * \
        expert_parallel_size


def _leading(value: Any, out: list) -> None:
    if isinstance(value, torch.Tensor) and value.ndim > 0:
        out.append(value)
    elif isinstance(value, Mapping):
        for v in value.values():
            _leading(v, out)
    elif is_dataclass(value) and not isinstance(value, type):
        for f in value.__dataclass_fields__:
            _leading(getattr(value, f), out)


def _slice(value: Any, a: int, b: int, n: int) -> Any:
    if isinstance(value, torch.Tensor):
        return value[a:b] if value.ndim > 0 and value.shape[0] == n else value
    if isinstance(value, Mapping):
        return type(value)((k, _slice(v, a, b, n)) for k, v in value.items())
    if isinstance(value, tuple) and hasattr(value, "_fields"):
        return type(value)(*(_slice(v, a, b, n) for v in value))
    if isinstance(value, Sequence) and not isinstance(value, (str, bytes)):
        return type(value)(_slice(v, a, b, n) for v in value)
    if is_dataclass(value) and not isinstance(value, type):
        return replace(value, **{f: _slice(getattr(value, f), a, b, n)
                                 for f in value.__dataclass_fields__})
    return value


def split_microbatches(batch: Any, micro_batch_size: int) -> tuple[Any, ...]:
    if micro_batch_size < 1:
        raise ValueError("micro_batch_size must be positive")
    tensors: list = []
    _leading(batch, tensors)
    if not tensors:
        raise ValueError("batch contains no tensor with a leading batch dimension")
    n = tensors[0].shape[0]
    if any(t.shape[0] != n for t in tensors):
        raise ValueError("all batched tensors must share the same leading dimension")
    if n % micro_batch_size:
        raise ValueError(f"batch size {n} is not divisible by micro_batch_size "
                         f"{micro_batch_size}")
    return tuple(_slice(batch, i, i + micro_batch_size, n) for i in range(0, n, micro_batch_size))
