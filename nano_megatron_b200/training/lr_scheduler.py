"""Learning-rate schedule keyed by the number of *completed* optimizer updates.

The rate installed after k completed updates is used by update k+1:
linear warmup ``base * (k+1) / W`` for k < W, then constant or cosine decay
from ``base`` to ``min_lr`` over ``decay_steps`` (default ``max_steps``).
Same schedule and checkpoint keys as the reference
(src/nano_megatron/training/lr_scheduler.py:14-128).
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from typing import Any


class LearningRateScheduler:
    STATE_VERSION = 1

    def __init__(self, *, config, optimizer_config, data_parallel, max_steps: int) -> None:
        self.schedule = str(getattr(config.schedule, "value", config.schedule)).lower()
        if self.schedule not in ("constant", "cosine"):
            raise ValueError(f"unsupported learning-rate schedule: {self.schedule!r}")
        self.base_lr = float(optimizer_config.lr)
        self.min_lr = float(config.min_lr)
        self.warmup_steps = int(config.warmup_steps)
        self.decay_steps = int(config.decay_steps or max_steps)
        if self.warmup_steps < 0:
            raise ValueError("warmup_steps must be non-negative")
        if self.decay_steps < 1:
            raise ValueError("decay_steps must be positive")
        if self.warmup_steps > self.decay_steps:
            raise ValueError("warmup_steps cannot exceed decay_steps")
        if not 0.0 <= self.min_lr <= self.base_lr:
            raise ValueError("min_lr must be between zero and the optimizer base LR")
        self.data_parallel = data_parallel
        self.completed_steps = 0
        self._apply()

    def rate_at(self, k: int) -> float:
        if isinstance(k, bool) or not isinstance(k, int):
            raise TypeError("completed_steps must be an integer")
        if k < 0:
            raise ValueError("completed_steps must be non-negative")
        if self.warmup_steps and k < self.warmup_steps:
            return self.base_lr * (k + 1) / self.warmup_steps
        if self.schedule == "constant":
            return self.base_lr
        span = self.decay_steps - self.warmup_steps
        if span <= 0:
            return self.min_lr if k >= self.decay_steps else self.base_lr
        t = min(1.0, max(0.0, (k - self.warmup_steps) / span))
        return self.min_lr + (self.base_lr - self.min_lr) * 0.5 * (1.0 + math.cos(math.pi * t))

    @property
    def learning_rate(self) -> float:
        return self.rate_at(self.completed_steps)

    def _apply(self) -> float:
        lr = self.learning_rate
        if self.data_parallel is not None:
            self.data_parallel.set_learning_rate(lr)
        return lr

    def set_completed_steps(self, k: int) -> float:
        if int(k) < 0:
            raise ValueError("completed_steps must be non-negative")
        self.completed_steps = int(k)
        return self._apply()

    def step(self) -> float:
        return self.set_completed_steps(self.completed_steps + 1)

    def state_dict(self) -> dict[str, Any]:
        return {"version": self.STATE_VERSION, "schedule": self.schedule,
                "base_lr": self.base_lr, "min_lr": self.min_lr,
                "warmup_steps": self.warmup_steps, "decay_steps": self.decay_steps,
                "completed_steps": self.completed_steps, "learning_rate": self.learning_rate}

    def load_state_dict(self, state: Mapping[str, Any], *,
                        expected_completed_steps: int | None = None) -> None:
        version = int(state.get("version", self.STATE_VERSION))
        if version != self.STATE_VERSION:
            raise ValueError(f"unsupported LR scheduler state version: {version}")
        for name in ("schedule", "base_lr", "min_lr", "warmup_steps", "decay_steps"):
            saved, now = state.get(name, getattr(self, name)), getattr(self, name)
            if saved != now:
                raise RuntimeError(f"LR scheduler configuration changed across resume for "
                                   f"{name}: {saved!r} != {now!r}")
        k = int(state.get("completed_steps", 0))
        if expected_completed_steps is not None and k != expected_completed_steps:
            raise RuntimeError("LR scheduler step does not match TrainerState.step: "
                               f"{k} != {expected_completed_steps}")
        self.set_completed_steps(k)
