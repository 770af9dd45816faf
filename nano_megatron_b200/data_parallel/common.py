"""Gradient-norm bookkeeping shared by the data-parallel strategies.

Counting rule of the reference (src/nano_megatron/data_parallel/_common.py:123-224):
a parameter contributes to the global norm once — TP-replicated parameters
only on TP rank 0, tied embedding copies only on their source rank, dense
(expert-replicated) parameters only on EP rank 0 — then the squared norm is summed
over TP x EP and PP (and, first, over the replica group when the gradient is
sharded, ZeRO; there the dense part is dropped on EP ranks other than 0 after that
sum, src/nano_megatron/data_parallel/_zero.py:137-151). The norm and the clip coefficient
``min(1, max_norm / (norm + 1e-6))`` stay on the device: nothing here
synchronises with the host.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from nano_megatron_b200.ops import functional as F
from nano_megatron_b200.parallel.group_plan import GroupKey


def counts_toward_norm(slice_, parallel) -> bool:
    if parallel is None:
        return True
    if not slice_.tensor_sharded and parallel.tp.size > 1 and parallel.tp.rank != 0:
        return False
    src = slice_.tied_source_rank
    if src is not None and parallel.rank != src:
        return False
    return True


def is_dense(bucket) -> bool:
    d = getattr(bucket, "domain", "dense")
    return str(getattr(d, "value", d)) == "dense"


def dense_counted_here(parallel) -> bool:
    """Dense parameters are replicated over EP: only EP rank 0 counts them."""
    ep = getattr(parallel, "ep", None) if parallel is not None else None
    return ep is None or ep.size == 1 or ep.rank == 0


def norm_ranges(buffers, parallel) -> list[tuple[int, int]]:
    """Merged [start, end) ranges of the flat (unsharded) gradient buffer that count toward
    the norm."""
    ranges: list[list[int]] = []
    dense_here = dense_counted_here(parallel)
    for bucket, s in buffers.slices():
        if not counts_toward_norm(s, parallel) or (is_dense(bucket) and not dense_here):
            continue
        a, b = bucket.offset + s.start, bucket.offset + s.end
        if ranges and ranges[-1][1] >= a - 8:
            ranges[-1][1] = b
        else:
            ranges.append([a, b])
    return [(a, b) for a, b in ranges]


def local_sumsq(flat: torch.Tensor, ranges) -> torch.Tensor:
    if not ranges:
        return torch.zeros((), device=flat.device, dtype=torch.float32)
    if len(ranges) == 1:
        return F.sumsq(flat[ranges[0][0]:ranges[0][1]])
    parts = [flat[a:b] for a, b in ranges]
    if flat.is_cuda:
        norms = torch._foreach_norm(parts)
        return torch.stack(norms).float().pow(2).sum()
    return sum(F.sumsq(p) for p in parts)


def reduce_model_parallel(sq: torch.Tensor, parallel) -> torch.Tensor:
    """Sum a squared norm over the TP x EP and PP groups."""
    if parallel is None:
        return sq
    for key in (GroupKey.TP_EP, GroupKey.PP):
        try:
            g = parallel.group(key)
        except KeyError:
            continue
        if g.size > 1:
            dist.all_reduce(sq, group=g.process_group)
    return sq


def clip_coefficient(total_norm: torch.Tensor, max_norm: float | None) -> torch.Tensor:
    if max_norm is None or max_norm <= 0:
        return torch.ones((), device=total_norm.device, dtype=torch.float32)
    return torch.clamp(max_norm / (total_norm.float() + 1e-6), max=1.0)
