"""Tensor-parallel linear layers (parameter holders with standalone forwards).

Parameter shapes, names and initialisation follow the reference
(src/nano_megatron/tensor_parallel/layers.py:27-214): column-parallel weights
are ``[out/TP, in]`` inside an ``nn.Linear`` called ``linear`` (Kaiming-uniform
on the local shard), row-parallel weights ``[out, in/TP]`` with a replicated,
zero-initialised bias applied after the reduction, the vocabulary-parallel LM
head ``[V/TP, H]`` (normal(0, init_std)) optionally sharing the embedding
Parameter.

Inside GPT layers these weights are consumed by the fused layer functions in
:mod:`nano_megatron_b200.models.gpt.blocks`; ``forward`` here is the generic
autograd path (used by tests and by anyone composing the layers directly).
"""

from __future__ import annotations

import torch
from torch import nn

from nano_megatron_b200.ops import functional as F

from .comm import (
    copy_to_tensor_parallel_region,
    gather_from_sequence_parallel_region,
    gather_from_tensor_parallel_region,
    reduce_from_tensor_parallel_region,
    reduce_scatter_to_sequence_parallel_region,
    scatter_to_tensor_parallel_region,
)


def tensor_parallel_group(parallel):
    """Accept a ParallelContext (use its TP group) or a group directly."""
    return parallel.tp if hasattr(parallel, "tp") and not hasattr(parallel, "ranks") else parallel


class _LinearFn(torch.autograd.Function):
    """y = x W^T on this library's GEMM (CPU: torch formula)."""

    @staticmethod
    def forward(ctx, x, weight):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        ctx.save_for_backward(x2, weight)
        ctx.shape = shape
        return F.linear(x2, weight).view(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, weight.shape[0]).contiguous()
        dx = F.linear_dgrad(dy2, weight).view(ctx.shape) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            acc = torch.zeros(weight.shape, dtype=torch.float32 if weight.dtype != torch.float64
                              else torch.float64, device=weight.device)
            F.linear_wgrad(dy2, x2, acc)
            dw = acc.to(weight.dtype)
        return dx, dw


def linear_forward(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None):
    y = _LinearFn.apply(x, weight)
    return y if bias is None else y + bias


class ColumnParallelLinear(nn.Module):
    """Weight sharded along the output features: ``[out/TP, in]``."""

    def __init__(self, in_features: int, out_features: int, *, parallel, kernels=None,
                 bias: bool = True, gather_output: bool = False, sequence_parallel: bool = False,
                 disable_input_gradient_reduce: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        if out_features % self.group.size:
            raise ValueError(f"out_features ({out_features}) must be divisible by TP size "
                             f"({self.group.size})")
        self.in_features = in_features
        self.out_features = out_features
        self.output_size_per_partition = out_features // self.group.size
        self.gather_output = gather_output
        self.sequence_parallel = sequence_parallel
        self.disable_input_gradient_reduce = disable_input_gradient_reduce
        self.linear = nn.Linear(in_features, self.output_size_per_partition, bias=bias,
                                device=device, dtype=dtype)

    weight = property(lambda self: self.linear.weight)
    bias = property(lambda self: self.linear.bias)

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0):
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected input hidden size {self.in_features}, got {x.shape[-1]}")
        if self.sequence_parallel:
            x = gather_from_sequence_parallel_region(x, self.group, sequence_dim=sequence_dim)
        elif not self.disable_input_gradient_reduce:
            x = copy_to_tensor_parallel_region(x, self.group)
        out = linear_forward(x, self.linear.weight, self.linear.bias)
        if self.gather_output:
            out = gather_from_tensor_parallel_region(out, self.group)
        return out, None


class RowParallelLinear(nn.Module):
    """Weight sharded along the input features: ``[out, in/TP]``; replicated bias."""

    def __init__(self, in_features: int, out_features: int, *, parallel, kernels=None,
                 bias: bool = True, input_is_parallel: bool = True,
                 sequence_parallel: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        if in_features % self.group.size:
            raise ValueError(f"in_features ({in_features}) must be divisible by TP size "
                             f"({self.group.size})")
        self.in_features = in_features
        self.out_features = out_features
        self.input_size_per_partition = in_features // self.group.size
        self.input_is_parallel = input_is_parallel
        self.sequence_parallel = sequence_parallel
        self.linear = nn.Linear(self.input_size_per_partition, out_features, bias=False,
                                device=device, dtype=dtype)
        self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) \
            if bias else None
        if self.bias is not None and sequence_parallel:
            self.bias.sequence_parallel_grad = True

    weight = property(lambda self: self.linear.weight)

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0):
        if self.input_is_parallel:
            if x.shape[-1] != self.input_size_per_partition:
                raise ValueError("parallel input must have local hidden size "
                                 f"{self.input_size_per_partition}, got {x.shape[-1]}")
        else:
            x = scatter_to_tensor_parallel_region(x, self.group)
        out = linear_forward(x, self.linear.weight)
        if self.sequence_parallel:
            out = reduce_scatter_to_sequence_parallel_region(out, self.group,
                                                             sequence_dim=sequence_dim)
        else:
            out = reduce_from_tensor_parallel_region(out, self.group)
        if self.bias is not None:
            out = out + self.bias
        return out, None


class VocabParallelLinear(nn.Module):
    """LM head ``[V/TP, H]`` (may share the embedding Parameter)."""

    def __init__(self, hidden_size: int, vocab_size: int, *, parallel, bias: bool = False,
                 sequence_parallel: bool = False, weight: nn.Parameter | None = None,
                 init_std: float = 0.02, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        if vocab_size % self.group.size:
            raise ValueError(f"vocab_size ({vocab_size}) must be divisible by TP size "
                             f"({self.group.size})")
        self.hidden_size = hidden_size
        self.vocab_size = vocab_size
        self.vocab_size_per_partition = vocab_size // self.group.size
        self.sequence_parallel = sequence_parallel
        if weight is None:
            self.weight = nn.Parameter(torch.empty(self.vocab_size_per_partition, hidden_size,
                                                   device=device, dtype=dtype))
            nn.init.normal_(self.weight, mean=0.0, std=init_std)
        else:
            expected = (self.vocab_size_per_partition, hidden_size)
            if tuple(weight.shape) != expected:
                raise ValueError(f"tied weight must have shape {expected}, got "
                                 f"{tuple(weight.shape)}")
            self.weight = weight
        self.bias = nn.Parameter(torch.zeros(self.vocab_size_per_partition, device=device,
                                             dtype=dtype)) if bias else None

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0) -> torch.Tensor:
        if x.shape[-1] != self.hidden_size:
            raise ValueError(f"expected input hidden size {self.hidden_size}, got {x.shape[-1]}")
        if self.sequence_parallel:
            x = gather_from_sequence_parallel_region(x, self.group, sequence_dim=sequence_dim)
        else:
            x = copy_to_tensor_parallel_region(x, self.group)
        return linear_forward(x, self.weight, self.bias)
