"""Tensor-parallel linear layers: parameter holders with a standalone autograd forward.

In the GPT layers the weights below are read by the fused layer functions of
:mod:`nano_megatron_b200.models.gpt.blocks` (GEMMs with their TP collectives fused in);
the ``forward`` methods here are the composable path for anyone who uses the layers on
their own, and for the tests.

Each layer is described by two things: which weight dim is split over the TP ranks, and
which collective sits on its input and on its output. Both are fixed at construction:

=====================  ==============  =============================  =======================
layer                  local weight    input                          output
=====================  ==============  =============================  =======================
ColumnParallelLinear   [out/TP, in]    SP: all-gather rows;           local columns (or
                                       else identity fwd / sum bwd    all-gathered)
RowParallelLinear      [out, in/TP]    already split (or split here)  SP: reduce-scatter rows;
                                                                      else all-reduce; + bias
VocabParallelLinear    [V/TP, H]       as ColumnParallelLinear        local vocabulary logits
=====================  ==============  =============================  =======================

Parameter names (``linear.weight`` inside an ``nn.Linear`` for column/row layers, a bare
``weight`` for the LM head), shapes and initialisation (the ``nn.Linear`` default on the
local shard, a zero replicated row bias, normal(0, init_std) LM head) are those of the
reference's layers (src/nano_megatron/tensor_parallel/layers.py), whose checkpoints use
these names.
"""

from __future__ import annotations

import torch
from torch import nn

from nano_megatron_b200.ops import functional as F

from . import comm as C


def tensor_parallel_group(parallel):
    """The TP group of a ParallelContext, or ``parallel`` itself when it is a group."""
    is_context = hasattr(parallel, "tp") and not hasattr(parallel, "ranks")
    return parallel.tp if is_context else parallel


def _split(total: int, parts: int, what: str) -> int:
    if total % parts:
        raise ValueError(f"{what}={total} does not split evenly over {parts} TP ranks")
    return total // parts


class _LinearFn(torch.autograd.Function):
    """``y = x @ W.T`` on this library's GEMM kernels (CPU: the torch formula); the weight
    gradient accumulates in fp32 before it is cast to the weight dtype."""

    @staticmethod
    def forward(ctx, x, weight):
        lead = x.shape[:-1]
        rows = x.reshape(-1, x.shape[-1]).contiguous()
        ctx.save_for_backward(rows, weight)
        ctx.lead = lead
        return F.linear(rows, weight).view(*lead, weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        rows, weight = ctx.saved_tensors
        dy_rows = dy.reshape(-1, weight.shape[0]).contiguous()
        want_x, want_w = ctx.needs_input_grad[:2]
        dx = F.linear_dgrad(dy_rows, weight).view(*ctx.lead, weight.shape[1]) if want_x else None
        dw = None
        if want_w:
            acc_dtype = torch.float64 if weight.dtype == torch.float64 else torch.float32
            acc = weight.new_zeros(weight.shape, dtype=acc_dtype)
            F.linear_wgrad(dy_rows, rows, acc)
            dw = acc.to(weight.dtype)
        return dx, dw


def linear_forward(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None):
    y = _LinearFn.apply(x, weight)
    return y if bias is None else y + bias


def _column_input(x, group, sequence_parallel: bool, skip_grad_reduce: bool, seq_dim: int):
    """The full-width input a column-split GEMM needs on every rank."""
    if sequence_parallel:
        return C.gather_from_sequence_parallel_region(x, group, sequence_dim=seq_dim)
    if skip_grad_reduce:
        return x
    return C.copy_to_tensor_parallel_region(x, group)


def _check_width(x: torch.Tensor, width: int, what: str) -> None:
    if x.shape[-1] != width:
        raise ValueError(f"{what}: last input dim is {x.shape[-1]}, expected {width}")


class ColumnParallelLinear(nn.Module):
    """Output features split over TP: local weight ``[out/TP, in]``."""

    def __init__(self, in_features: int, out_features: int, *, parallel, kernels=None,
                 bias: bool = True, gather_output: bool = False, sequence_parallel: bool = False,
                 disable_input_gradient_reduce: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        self.in_features, self.out_features = in_features, out_features
        self.output_size_per_partition = _split(out_features, self.group.size, "out_features")
        self.gather_output = gather_output
        self.sequence_parallel = sequence_parallel
        self.disable_input_gradient_reduce = disable_input_gradient_reduce
        self.linear = nn.Linear(in_features, self.output_size_per_partition, bias=bias,
                                device=device, dtype=dtype)

    @property
    def weight(self):
        return self.linear.weight

    @property
    def bias(self):
        return self.linear.bias

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0):
        _check_width(x, self.in_features, "ColumnParallelLinear")
        full = _column_input(x, self.group, self.sequence_parallel,
                             self.disable_input_gradient_reduce, sequence_dim)
        y = linear_forward(full, self.linear.weight, self.linear.bias)
        if self.gather_output:
            y = C.gather_from_tensor_parallel_region(y, self.group)
        return y, None


class RowParallelLinear(nn.Module):
    """Input features split over TP: local weight ``[out, in/TP]``; the bias is replicated
    and added once, after the partial products are summed."""

    def __init__(self, in_features: int, out_features: int, *, parallel, kernels=None,
                 bias: bool = True, input_is_parallel: bool = True,
                 sequence_parallel: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        self.in_features, self.out_features = in_features, out_features
        self.input_size_per_partition = _split(in_features, self.group.size, "in_features")
        self.input_is_parallel = input_is_parallel
        self.sequence_parallel = sequence_parallel
        self.linear = nn.Linear(self.input_size_per_partition, out_features, bias=False,
                                device=device, dtype=dtype)
        self.bias = None
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype))
            # under SP each rank sees 1/TP of the rows: the bias gradient is summed over TP
            self.bias.sequence_parallel_grad = bool(sequence_parallel)

    @property
    def weight(self):
        return self.linear.weight

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0):
        if self.input_is_parallel:
            _check_width(x, self.input_size_per_partition, "RowParallelLinear (split input)")
        else:
            x = C.scatter_to_tensor_parallel_region(x, self.group)
        partial = linear_forward(x, self.linear.weight)
        if self.sequence_parallel:
            y = C.reduce_scatter_to_sequence_parallel_region(partial, self.group,
                                                             sequence_dim=sequence_dim)
        else:
            y = C.reduce_from_tensor_parallel_region(partial, self.group)
        return (y if self.bias is None else y + self.bias), None


class VocabParallelLinear(nn.Module):
    """LM head with the vocabulary split over TP: ``[V/TP, H]``. ``weight`` may be the
    embedding's Parameter (tied embeddings), which then must have that shape."""

    def __init__(self, hidden_size: int, vocab_size: int, *, parallel, bias: bool = False,
                 sequence_parallel: bool = False, weight: nn.Parameter | None = None,
                 init_std: float = 0.02, device=None, dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        self.hidden_size, self.vocab_size = hidden_size, vocab_size
        self.vocab_size_per_partition = _split(vocab_size, self.group.size, "vocab_size")
        self.sequence_parallel = sequence_parallel
        shape = (self.vocab_size_per_partition, hidden_size)
        if weight is not None and tuple(weight.shape) != shape:
            raise ValueError(f"shared LM-head weight has shape {tuple(weight.shape)}; this "
                             f"TP rank needs {shape}")
        if weight is None:
            weight = nn.Parameter(torch.empty(shape, device=device, dtype=dtype))
            nn.init.normal_(weight, mean=0.0, std=init_std)
        self.weight = weight
        self.bias = nn.Parameter(torch.zeros(shape[0], device=device, dtype=dtype)) \
            if bias else None

    def forward(self, x: torch.Tensor, *, sequence_dim: int = 0) -> torch.Tensor:
        _check_width(x, self.hidden_size, "VocabParallelLinear")
        full = _column_input(x, self.group, self.sequence_parallel, False, sequence_dim)
        return linear_forward(full, self.weight, self.bias)
