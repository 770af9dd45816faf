"""Token-weighted loss metrics.

The last pipeline stage sums (loss_sum, token_count) over DENSE_REPLICA in
fp64 and broadcasts them over PP so every rank reports the same value
(reference: src/nano_megatron/training/metrics.py:15-122). Values stay on the
device.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from nano_megatron_b200.parallel.group_plan import GroupKey


class MetricStore:
    def __init__(self) -> None:
        self.values: dict[str, list[float]] = {}

    def add(self, name: str, value: float) -> None:
        self.values.setdefault(name, []).append(float(value))

    def mean(self, name: str) -> float:
        v = self.values.get(name, [])
        return sum(v) / len(v) if v else float("nan")

    def clear(self) -> None:
        self.values.clear()


def aggregate_loss_metrics(acc, parallel, device):
    stats = torch.zeros(2, dtype=torch.float64, device=device)
    if acc is not None and acc.loss_sum is not None:
        stats[0] = acc.loss_sum.to(device)
        stats[1] = acc.token_count.to(device)
    if parallel is not None and dist.is_available() and dist.is_initialized():
        g = parallel.group(GroupKey.DENSE_REPLICA)
        if g.size > 1:
            dist.all_reduce(stats, group=g.process_group)
        pp = parallel.pp
        if pp.size > 1:
            dist.broadcast(stats, src=pp.ranks[-1], group=pp.process_group)
    return stats[0], stats[1]


def loss_and_perplexity(loss_sum: float, token_count: float) -> tuple[float, float]:
    loss = loss_sum / max(token_count, 1.0)
    return loss, math.exp(min(loss, 50.0))
