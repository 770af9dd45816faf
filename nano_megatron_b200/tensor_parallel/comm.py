"""Tensor-parallel collectives and their autograd "region" wrappers.

Activations inside this framework are sequence-major (``[S, B, H]`` flattened
to ``[S*B, H]``), so a sequence-parallel shard is a contiguous block of rows
and the SP all-gather / reduce-scatter are plain contiguous NCCL collectives
(no permutes). The region functions keep the reference's names and semantics
(src/nano_megatron/tensor_parallel/sequence_parallel.py:21-204) and take a
``sequence_dim`` argument.

On CUDA the fused sm_100a paths (all-gather->GEMM, GEMM->reduce-scatter over
NVLink peer memory) replace these calls inside the model's layer functions;
these NCCL forms remain the generic path and the reference the fused kernels
are tested against.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _pg(group):
    return getattr(group, "process_group", None)


def all_reduce(x: torch.Tensor, group, op=dist.ReduceOp.SUM) -> torch.Tensor:
    if group is None or group.size == 1:
        return x
    dist.all_reduce(x, op=op, group=_pg(group))
    return x


def all_gather_dim0(x: torch.Tensor, group) -> torch.Tensor:
    """Concatenate every rank's ``x`` along dim 0 (rank order)."""
    if group is None or group.size == 1:
        return x
    x = x.contiguous()
    out = torch.empty((group.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                      device=x.device)
    dist.all_gather_into_tensor(out, x, group=_pg(group))
    return out


def reduce_scatter_dim0(x: torch.Tensor, group) -> torch.Tensor:
    """Sum over ranks, keep this rank's 1/size block of dim 0."""
    if group is None or group.size == 1:
        return x
    x = x.contiguous()
    if x.shape[0] % group.size:
        raise ValueError(f"dim 0 ({x.shape[0]}) must be divisible by group size {group.size}")
    out = torch.empty((x.shape[0] // group.size,) + tuple(x.shape[1:]), dtype=x.dtype,
                      device=x.device)
    if x.device.type == "cpu" and dist.get_backend(_pg(group)) == "gloo":
        # gloo has no reduce_scatter: all-reduce then slice
        full = x.clone()
        dist.all_reduce(full, group=_pg(group))
        n = out.shape[0]
        out.copy_(full[group.rank * n:(group.rank + 1) * n])
        return out
    dist.reduce_scatter_tensor(out, x, group=_pg(group))
    return out


def _move(x: torch.Tensor, dim: int) -> torch.Tensor:
    return x if dim == 0 else x.movedim(dim, 0)


def gather_along(x: torch.Tensor, group, dim: int) -> torch.Tensor:
    if group is None or group.size == 1:
        return x
    return _move(all_gather_dim0(_move(x, dim).contiguous(), group), dim) if dim else \
        all_gather_dim0(x, group)


def reduce_scatter_along(x: torch.Tensor, group, dim: int) -> torch.Tensor:
    if group is None or group.size == 1:
        return x
    if dim == 0:
        return reduce_scatter_dim0(x, group)
    return reduce_scatter_dim0(x.movedim(dim, 0).contiguous(), group).movedim(0, dim)


def split_along(x: torch.Tensor, group, dim: int) -> torch.Tensor:
    if group is None or group.size == 1:
        return x
    n = x.shape[dim] // group.size
    return x.narrow(dim, group.rank * n, n).contiguous()


class _Copy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return all_reduce(g.contiguous().clone(), ctx.group), None


class _Reduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        return all_reduce(x.contiguous().clone(), group)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _Scatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return split_along(x, group, dim)

    @staticmethod
    def backward(ctx, g):
        return gather_along(g.contiguous(), ctx.group, ctx.dim), None, None


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return gather_along(x.contiguous(), group, dim)

    @staticmethod
    def backward(ctx, g):
        return split_along(g, ctx.group, ctx.dim), None, None


class _SeqGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return gather_along(x.contiguous(), group, dim)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_along(g.contiguous(), ctx.group, ctx.dim), None, None


class _SeqReduceScatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return reduce_scatter_along(x.contiguous(), group, dim)

    @staticmethod
    def backward(ctx, g):
        return gather_along(g.contiguous(), ctx.group, ctx.dim), None, None


def copy_to_tensor_parallel_region(x, group):
    """Identity forward, all-reduce of the gradient in backward."""
    return x if group.size == 1 else _Copy.apply(x, group)


def reduce_from_tensor_parallel_region(x, group):
    """All-reduce forward, identity backward."""
    return x if group.size == 1 else _Reduce.apply(x, group)


def scatter_to_tensor_parallel_region(x, group, dim: int = -1):
    return x if group.size == 1 else _Scatter.apply(x, group, dim % x.dim())


def gather_from_tensor_parallel_region(x, group, dim: int = -1):
    return x if group.size == 1 else _Gather.apply(x, group, dim % x.dim())


def gather_from_sequence_parallel_region(x, group, *, sequence_dim: int = 0):
    """All-gather along the sequence dimension; reduce-scatter in backward."""
    return x if group.size == 1 else _SeqGather.apply(x, group, sequence_dim % x.dim())


def reduce_scatter_to_sequence_parallel_region(x, group, *, sequence_dim: int = 0):
    """Reduce-scatter along the sequence dimension; all-gather in backward."""
    return x if group.size == 1 else _SeqReduceScatter.apply(x, group, sequence_dim % x.dim())


def scatter_to_sequence_parallel_region(x, group, *, sequence_dim: int = 0):
    """Keep this rank's block of the sequence dimension (no reduction: the input is
    replicated over the group); all-gather in backward."""
    return x if group.size == 1 else _Scatter.apply(x, group, sequence_dim % x.dim())


_SP_HOOKED = "_nmb_sequence_parallel_hooked"


def register_sequence_parallel_gradient_hooks(module, group, *, recurse: bool = True) -> None:
    """Sum, over the group, the gradients of ``module``'s parameters that are replicated
    across sequence-parallel ranks (norm weights, biases of row-parallel layers): each rank
    saw only its sequence block, so the full gradient is the sum.

    For modules trained through ``.grad`` (plain autograd): a post-accumulate hook
    all-reduces each parameter's gradient as soon as autograd has finished it. Registering
    twice for the same parameter and group is a no-op. The fused GPT blocks of this
    framework accumulate into ``main_grad`` instead and sum these gradients once per step
    in the data-parallel strategy (``_reduce_sequence_parallel_grads``), without hooks.
    """
    if group is None or group.size == 1:
        return
    pg = _pg(group)
    for p in module.parameters(recurse=recurse):
        seen = getattr(p, _SP_HOOKED, None)
        if seen is None:
            seen = set()
            setattr(p, _SP_HOOKED, seen)
        if id(pg) in seen:
            continue
        seen.add(id(pg))

        def _sum_over_sequence_ranks(param, _pg=pg):
            if param.grad is not None:
                dist.all_reduce(param.grad, group=_pg)

        p.register_post_accumulate_grad_hook(_sum_over_sequence_ranks)
