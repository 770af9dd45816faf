"""Vocabulary-parallel cross-entropy.

The reference (src/nano_megatron/tensor_parallel/cross_entropy.py:30-123) runs
three fp32 all-reduces (max, target logit, sum-exp) and keeps the full softmax
for backward. Here each rank computes per-row (max, sum-exp, target) for its
shard in one kernel, the ranks exchange those 3 floats per row in ONE
all-gather, and a second kernel merges them into the loss and writes the local
``softmax - onehot`` gradient in place of the logits (no fp32 softmax copy is
kept). ignore_index is -100 (any negative label is ignored); reduction
``mean`` over valid tokens or ``sum``/``none``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from nano_megatron_b200.ops import functional as F

from .layers import tensor_parallel_group

IGNORE_INDEX = -100


def vocab_parallel_ce_rows(logits2d: torch.Tensor, labels1d: torch.Tensor, group,
                           write_grad: bool) -> torch.Tensor:
    """Per-row loss; when ``write_grad`` the logits are overwritten by d loss_row / d logits."""
    if group is None or group.size == 1:
        return F.ce_local(logits2d, labels1d, write_grad)
    vstart = group.rank * logits2d.shape[1]
    stats = F.ce_stats(logits2d, labels1d, vstart)
    gathered = torch.empty((group.size * stats.shape[0],) + tuple(stats.shape[1:]),
                           dtype=stats.dtype, device=stats.device)
    dist.all_gather_into_tensor(gathered, stats.contiguous(), group=group.process_group)
    return F.ce_finish(logits2d, labels1d, vstart, gathered.view(group.size, *stats.shape),
                       write_grad)


class _VocabParallelCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, group, reduction, original_vocab_size):
        shape = labels.shape
        l2 = logits.reshape(-1, logits.shape[-1])
        work = l2.detach().clone() if l2.dtype != torch.float32 or True else l2
        lab = labels.reshape(-1).to(torch.long)
        rows = vocab_parallel_ce_rows(work, lab, group, write_grad=True)
        valid = (lab >= 0).to(rows.dtype)
        count = valid.sum()
        ctx.reduction = reduction
        ctx.shape = logits.shape
        ctx.save_for_backward(work, count)
        if reduction == "mean":
            return rows.sum() / count.clamp_min(1)
        if reduction == "sum":
            return rows.sum()
        return rows.view(shape)

    @staticmethod
    def backward(ctx, g):
        work, count = ctx.saved_tensors
        if ctx.reduction == "mean":
            grad = work.float() * (g / count.clamp_min(1))
        elif ctx.reduction == "sum":
            grad = work.float() * g
        else:
            grad = work.float() * g.reshape(-1, 1)
        return grad.to(work.dtype).view(ctx.shape), None, None, None, None


class VocabParallelCrossEntropy(nn.Module):
    def __init__(self, *, parallel, reduction: str = "mean", ignore_index: int = IGNORE_INDEX,
                 original_vocab_size: int | None = None) -> None:
        super().__init__()
        if reduction not in ("mean", "sum", "none"):
            raise ValueError("reduction must be mean, sum or none")
        if ignore_index != IGNORE_INDEX:
            raise ValueError("only ignore_index=-100 is supported")
        self.group = tensor_parallel_group(parallel)
        self.reduction = reduction
        self.original_vocab_size = original_vocab_size

    def forward(self, logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return _VocabParallelCEFn.apply(logits, labels, self.group, self.reduction,
                                        self.original_vocab_size)
