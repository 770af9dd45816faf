"""Gradient accumulation without pipeline parallelism (PP = 1)."""

from __future__ import annotations

import torch

from .base import LossAccumulator, extract_loss


class NoPipelineSchedule:
    def __init__(self, stage, data_parallel) -> None:
        self.stage = stage
        self.data_parallel = data_parallel

    def forward_backward(self, microbatches, *, forward_only: bool = False
                         ) -> LossAccumulator:
        acc = LossAccumulator()
        m = len(microbatches)
        dp = self.data_parallel
        for i, mb in enumerate(microbatches):
            last = i == m - 1
            if forward_only:
                with torch.no_grad():
                    extract_loss(self.stage(None, mb), mb, m, acc)
                continue
            with dp.forward_microbatch_context(synchronize_gradients=last):
                loss = extract_loss(self.stage(None, mb), mb, m, acc)
            with dp.microbatch_context(is_last_microbatch=last):
                dp.backward(loss)
        return acc
