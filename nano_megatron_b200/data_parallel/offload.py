"""Offload policy: activations to pinned host memory; optimizer state on host.

Reference: src/nano_megatron/data_parallel/offload.py:11-112.
"""

from __future__ import annotations

from contextlib import contextmanager, nullcontext
from dataclasses import dataclass

import torch

from nano_megatron_b200.nn.activation_checkpoint import ActivationOffloadHooks


@dataclass(frozen=True)
class OffloadPolicy:
    optimizer_state: bool = False
    zero3_params_and_grads: bool = False
    activations: bool = False
    pin_memory: bool = True
    non_blocking: bool = True

    @classmethod
    def from_config(cls, config) -> "OffloadPolicy":
        if config is None:
            return cls()
        return cls(**{k: bool(getattr(config, k, getattr(cls, k))) for k in
                      ("optimizer_state", "zero3_params_and_grads", "activations", "pin_memory",
                       "non_blocking")})

    def validate(self, mode: str) -> None:
        if self.optimizer_state and mode not in ("zero1", "zero2"):
            raise ValueError("optimizer-state offload requires data_parallel.mode zero1 or zero2")
        if self.zero3_params_and_grads and mode != "zero3":
            raise ValueError("offload.zero3_params_and_grads requires data_parallel.mode=zero3")


class ActivationOffloader:
    def __init__(self, policy: OffloadPolicy) -> None:
        self.policy = policy

    @contextmanager
    def context(self):
        ctx = ActivationOffloadHooks(self.policy.pin_memory) if self.policy.activations \
            else nullcontext()
        with ctx:
            yield


class OptimizerStateStorage:
    """Allocate optimizer state on the device or in pinned host memory."""

    def __init__(self, policy: OffloadPolicy, device: torch.device) -> None:
        self.offload = policy.optimizer_state
        self.device = device
        self.pin = policy.pin_memory

    def zeros(self, n: int) -> torch.Tensor:
        if self.offload:
            return torch.zeros(n, dtype=torch.float32, pin_memory=self.pin and torch.cuda.is_available())
        return torch.zeros(n, dtype=torch.float32, device=self.device)
