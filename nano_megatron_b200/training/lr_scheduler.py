"""Learning-rate schedule as a pure function of the number of completed optimizer updates.

A :class:`ScheduleSpec` is the whole schedule (kind, base and floor rate, warmup and
decay horizon); ``spec.rate(k)`` is the rate that update ``k + 1`` applies, i.e. the
rate installed after ``k`` completed updates:

* warmup (``k < warmup``): ramps linearly, ``base * (k + 1) / warmup``;
* afterwards ``constant`` stays at ``base``; ``cosine`` follows half a cosine period
  from ``base`` (at ``k = warmup``) to ``min_lr`` (at ``k = decay``) and stays there.

Because the rate depends only on ``k``, restoring a checkpoint is installing
``spec.rate(step)``; the scheduler's checkpoint entry records the spec so a resume
with a different schedule is refused. The entry's keys are those the reference's
trainer state carries (src/nano_megatron/training/lr_scheduler.py:90-101), so
checkpoints move between the two frameworks.
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import astuple, dataclass, fields
from typing import Any

_KINDS = ("constant", "cosine")


@dataclass(frozen=True)
class ScheduleSpec:
    schedule: str
    base_lr: float
    min_lr: float
    warmup_steps: int
    decay_steps: int

    @classmethod
    def from_configs(cls, config, optimizer_config, max_steps: int) -> "ScheduleSpec":
        kind = str(getattr(config.schedule, "value", config.schedule)).lower()
        spec = cls(schedule=kind, base_lr=float(optimizer_config.lr),
                   min_lr=float(config.min_lr), warmup_steps=int(config.warmup_steps),
                   decay_steps=int(config.decay_steps or max_steps))
        spec.check()
        return spec

    def check(self) -> None:
        problems = []
        if self.schedule not in _KINDS:
            problems.append(f"schedule {self.schedule!r} is not one of {_KINDS}")
        if self.warmup_steps < 0:
            problems.append(f"warmup_steps={self.warmup_steps} is negative")
        if self.decay_steps < 1:
            problems.append(f"decay_steps={self.decay_steps} must be at least 1")
        elif self.warmup_steps > self.decay_steps:
            problems.append(f"warmup_steps={self.warmup_steps} is past "
                            f"decay_steps={self.decay_steps}")
        if self.min_lr < 0 or self.min_lr > self.base_lr:
            problems.append(f"min_lr={self.min_lr} lies outside [0, lr={self.base_lr}]")
        if problems:
            raise ValueError("invalid learning-rate schedule: " + "; ".join(problems))

    def rate(self, completed: int) -> float:
        if isinstance(completed, bool) or not isinstance(completed, int):
            raise TypeError(f"completed update count must be an int, got {completed!r}")
        if completed < 0:
            raise ValueError(f"completed update count {completed} is negative")
        w, d = self.warmup_steps, self.decay_steps
        if completed < w:
            return self.base_lr * (completed + 1) / w
        if self.schedule == "constant":
            return self.base_lr
        if d == w:                       # no decay phase: a step down at the horizon
            return self.base_lr if completed < d else self.min_lr
        frac = min(completed - w, d - w) / (d - w)
        return self.min_lr + 0.5 * (self.base_lr - self.min_lr) * (1.0 + math.cos(math.pi * frac))


class LearningRateScheduler:
    """Holds a :class:`ScheduleSpec` and the completed-update count; every change of the
    count installs the matching rate in the data-parallel strategy (which feeds it to the
    optimizer kernel on the device)."""

    STATE_VERSION = 1

    def __init__(self, *, config, optimizer_config, data_parallel, max_steps: int) -> None:
        self.spec = ScheduleSpec.from_configs(config, optimizer_config, max_steps)
        self.data_parallel = data_parallel
        self.completed_steps = 0
        self._install()

    # the spec's fields, readable as attributes of the scheduler
    schedule = property(lambda self: self.spec.schedule)
    base_lr = property(lambda self: self.spec.base_lr)
    min_lr = property(lambda self: self.spec.min_lr)
    warmup_steps = property(lambda self: self.spec.warmup_steps)
    decay_steps = property(lambda self: self.spec.decay_steps)

    def rate_at(self, completed: int) -> float:
        return self.spec.rate(completed)

    @property
    def learning_rate(self) -> float:
        return self.spec.rate(self.completed_steps)

    def _install(self) -> float:
        lr = self.learning_rate
        if self.data_parallel is not None:
            self.data_parallel.set_learning_rate(lr)
        return lr

    def set_completed_steps(self, completed: int) -> float:
        completed = int(completed)
        self.spec.rate(completed)        # validates the count before it is stored
        self.completed_steps = completed
        return self._install()

    def step(self) -> float:
        return self.set_completed_steps(self.completed_steps + 1)

    def state_dict(self) -> dict[str, Any]:
        entry: dict[str, Any] = {"version": self.STATE_VERSION}
        entry.update({f.name: getattr(self.spec, f.name) for f in fields(self.spec)})
        entry["completed_steps"] = self.completed_steps
        entry["learning_rate"] = self.learning_rate
        return entry

    def load_state_dict(self, state: Mapping[str, Any], *,
                        expected_completed_steps: int | None = None) -> None:
        version = int(state.get("version", self.STATE_VERSION))
        if version != self.STATE_VERSION:
            raise ValueError(f"learning-rate state has version {version}; this build reads "
                             f"version {self.STATE_VERSION}")
        saved = tuple(state.get(f.name, getattr(self.spec, f.name)) for f in fields(self.spec))
        if saved != astuple(self.spec):
            diff = [f"{f.name}: checkpoint {s!r}, config {c!r}"
                    for f, s, c in zip(fields(self.spec), saved, astuple(self.spec)) if s != c]
            raise RuntimeError("resumed run changes the learning-rate schedule (" +
                               ", ".join(diff) + ")")
        completed = int(state.get("completed_steps", 0))
        if expected_completed_steps is not None and completed != expected_completed_steps:
            raise RuntimeError(f"learning-rate state is at update {completed} but the trainer "
                               f"state is at step {expected_completed_steps}")
        self.set_completed_steps(completed)
