"""Tied input embedding / LM head across the first and last pipeline stages.

The EMBEDDING group holds the first and last PP stage of one TP/CP/EP/DP
coordinate. The first stage's weight is broadcast once before pipeline P2P
starts; the two endpoints' gradients are summed after the whole pipeline
backward (never from a hook, which could deadlock against P2P). Reference:
src/nano_megatron/models/gpt/tied_embeddings.py:15-118. Gradients live in the
parameter's fp32 ``main_grad``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class TiedEmbeddingSynchronizer:
    def __init__(self, weight: torch.nn.Parameter, group) -> None:
        if weight.ndim != 2:
            raise ValueError(f"a tied embedding shard must be a matrix, got shape "
                             f"{tuple(weight.shape)}")
        if group.size not in (1, 2):
            raise ValueError("the embedding group must contain the first and last pipeline "
                             f"stages; got {group.size} ranks")
        self.group = group
        self._shape = tuple(weight.shape)
        self._synced = group.size == 1
        self.bind_weight(weight)

    def bind_weight(self, weight) -> None:
        if tuple(weight.shape) != self._shape:
            raise ValueError("replacement tied embedding has a different global shape: "
                             f"expected {self._shape}, got {tuple(weight.shape)}")
        self.weight = weight
        weight._nano_megatron_tied_source_rank = self.source_rank

    @property
    def source_rank(self) -> int:
        ranks = getattr(self.group, "ranks", None)
        return int(ranks[0]) if ranks else 0

    @property
    def active(self) -> bool:
        return self.group.size > 1

    @property
    def weight_is_synchronized(self) -> bool:
        return self._synced

    def _pg(self):
        if not dist.is_available() or not dist.is_initialized() or self.group.process_group is None:
            raise RuntimeError("a multi-rank tied embedding group requires initialized "
                               "torch.distributed and a materialized process group")
        return self.group.process_group

    @torch.no_grad()
    def synchronize_weight(self, *, force: bool = False) -> None:
        if not self.active or (self._synced and not force):
            return
        dist.broadcast(self.weight.data, src=self.source_rank, group=self._pg())
        master = getattr(self.weight, "_fp32_master", None)
        if master is not None:
            dist.broadcast(master, src=self.source_rank, group=self._pg())
        self._synced = True

    @torch.no_grad()
    def synchronize_gradient(self) -> None:
        if not self.active:
            return
        grad = getattr(self.weight, "main_grad", None)
        if grad is None:
            grad = self.weight.grad
        if grad is None:
            grad = torch.zeros(self._shape, dtype=torch.float32, device=self.weight.device)
            self.weight.main_grad = grad
        dist.all_reduce(grad, group=self._pg())
