"""Schedule helpers shared by all pipeline schedules.

``extract_loss`` scales a microbatch loss by 1/M and accumulates the
token-weighted loss sum and token count ON THE DEVICE (the reference does a
host ``.cpu()`` per microbatch, src/nano_megatron/pipeline_parallel/schedules/
base.py:108-121).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class LossAccumulator:
    loss_sum: torch.Tensor | None = None
    token_count: torch.Tensor | None = None
    losses: list = field(default_factory=list)

    def add(self, loss: torch.Tensor, labels: torch.Tensor | None) -> None:
        d = loss.detach()
        if labels is not None:
            n = (labels >= 0).sum().to(device=d.device, dtype=torch.float64)
        else:
            n = torch.ones((), dtype=torch.float64, device=d.device)
        s = d.to(torch.float64) * n
        self.loss_sum = s if self.loss_sum is None else self.loss_sum + s
        self.token_count = n if self.token_count is None else self.token_count + n
        self.losses.append(d)


def batch_labels(batch):
    if isinstance(batch, dict):
        return batch.get("labels")
    return getattr(batch, "labels", None)


def extract_loss(output: torch.Tensor, batch, num_microbatches: int,
                 acc: LossAccumulator | None) -> torch.Tensor:
    if acc is not None:
        acc.add(output, batch_labels(batch))
    return output / num_microbatches


def forward_microbatch_context(data_parallel, *, synchronize_gradients: bool, unit=None):
    return data_parallel.forward_microbatch_context(synchronize_gradients=synchronize_gradients,
                                                    unit=unit)


def microbatch_context(data_parallel, *, is_last_microbatch: bool, unit=None):
    return data_parallel.microbatch_context(is_last_microbatch=is_last_microbatch, unit=unit)
