"""Optional Weights & Biases telemetry, layered over the local metric timeline.

Only the primary rank of a run with ``wandb.enabled`` (and a mode other than
``disabled``) talks to W&B, and ``wandb`` is imported only then; every rank that owns the
timeline writes ``metrics.jsonl`` regardless (:mod:`.metric_history`).

Run identity. A fresh run uses the configured ``run_id`` (which W&B may resume) or a new
one. A run resumed from a checkpoint never appends to the checkpoint's W&B run, whose
later points the checkpoint has not seen: it opens a new run (``resume="never"``, an id
different from the checkpoint's), logs into it the checkpoint's part of the timeline, and
records where it came from in the run summary (``wandb/logical_fork``,
``wandb/forked_from_step``, ``wandb/forked_from_run_id``,
``wandb/history_replayed_records``). The policy and those summary keys are the
reference's (src/nano_megatron/training/wandb_logger.py), so dashboards treat runs of both
frameworks alike.
"""

from __future__ import annotations

import importlib
import uuid
from collections.abc import Mapping
from dataclasses import fields, is_dataclass
from enum import Enum
from pathlib import Path
from typing import Any

from .metric_history import JsonlMetricHistory


def plain_config(v: Any) -> Any:
    """A config object as plain JSON-able data (dataclasses -> dicts, enums and paths ->
    strings), for the W&B run's config panel."""
    if isinstance(v, (Enum, Path)):
        return str(v.value if isinstance(v, Enum) else v)
    if is_dataclass(v) and not isinstance(v, type):
        v = {f.name: getattr(v, f.name) for f in fields(v)}
    if isinstance(v, Mapping):
        return {str(k): plain_config(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [plain_config(x) for x in v]
    return v


def _fresh_id(mod) -> str:
    make = getattr(getattr(mod, "util", None), "generate_id", None)
    made = make() if callable(make) else None
    return made if isinstance(made, str) and made else uuid.uuid4().hex


def _choose_run_id(mod, configured: str | None, source_run: str | None, forked: bool) -> str:
    if not forked:
        return configured or _fresh_id(mod)
    rid = configured if configured not in (None, source_run) else _fresh_id(mod)
    while rid == source_run:                # a generator that repeats the source's id
        rid = uuid.uuid4().hex
    return rid


class WandbLogger:
    def __init__(self, config, *, run_config, is_primary: bool, wandb_module=None,
                 metrics_path: Path | None = None, resume_metrics_path: Path | None = None) -> None:
        self.config = config
        self.run_config = run_config
        self.enabled = bool(is_primary and config is not None and config.enabled
                            and config.mode != "disabled")
        self._wandb = wandb_module
        self._run = None
        self.run_id: str | None = None
        self.history = JsonlMetricHistory(metrics_path, source=resume_metrics_path,
                                          enabled=is_primary)

    # ------------------------------------------------------------------ start
    def start(self, *, checkpoint_run_id: str | None = None, checkpoint_step: int | None = None,
              checkpoint_metrics_state: Mapping[str, Any] | None = None, model=None
              ) -> str | None:
        """Start the timeline and (primary, enabled) the W&B run; returns the run id."""
        if self._run is not None:
            return self.run_id
        forked = checkpoint_step is not None
        if forked:
            if type(checkpoint_step) is not int or checkpoint_step < 0:
                raise ValueError(f"checkpoint_step must be a non-negative int, got "
                                 f"{checkpoint_step!r}")
        elif checkpoint_run_id is not None:
            raise ValueError("a checkpoint_run_id without its checkpoint_step")
        replay = self.history.start(through_step=checkpoint_step,
                                    expected_state=checkpoint_metrics_state)
        if not self.enabled:
            return None
        mod = self._module()
        rid = _choose_run_id(mod, self.config.run_id, checkpoint_run_id, forked)
        self._run = mod.init(**self._init_options(rid, forked))
        if self._run is None:
            raise RuntimeError("wandb.init() gave no run object")
        got = getattr(self._run, "id", rid)
        if not (isinstance(got, str) and got):
            raise RuntimeError(f"W&B run id {got!r} is not a non-empty string")
        self.run_id = got
        self._declare_step_axis(mod)
        for rec in replay:
            self._run.log(rec.wandb_payload())
        summary: dict[str, Any] = {}
        if forked:
            summary.update({"wandb/logical_fork": True, "wandb/forked_from_step": checkpoint_step,
                            "wandb/history_replayed_records": len(replay)})
            if checkpoint_run_id is not None:
                summary["wandb/forked_from_run_id"] = checkpoint_run_id
        if self.history.destination is not None:
            summary["metrics/history_path"] = str(self.history.destination)
        if model is not None:
            sizes = [(p.numel(), p.requires_grad) for p in model.parameters()]
            summary["model/parameters"] = sum(n for n, _ in sizes)
            summary["model/trainable_parameters"] = sum(n for n, g in sizes if g)
        self.update_summary(summary)
        return self.run_id

    def _init_options(self, rid: str, forked: bool) -> dict[str, Any]:
        c = self.config
        opts = {"project": c.project, "entity": c.entity, "name": c.name, "group": c.group,
                "tags": list(c.tags), "mode": c.mode,
                "dir": str(c.directory) if c.directory is not None else None, "id": rid,
                "config": plain_config(self.run_config),
                "resume": "never" if forked else "allow"}
        return {k: v for k, v in opts.items() if v is not None}

    @staticmethod
    def _declare_step_axis(mod) -> None:
        define = getattr(mod, "define_metric", None)
        if not callable(define):
            return
        define("trainer/step")
        for family in ("train/*", "validation/*"):
            define(family, step_metric="trainer/step")

    # ------------------------------------------------------------------ logging
    def log(self, prefix: str, metrics: Mapping[str, float], *, state) -> None:
        rec = self.history.append(prefix, metrics, state=state)
        if self._run is None:
            return
        if rec is None:      # no local timeline on this rank: build the same row directly
            row = {"trainer/step": int(state.step),
                   "trainer/consumed_samples": int(state.consumed_samples),
                   "trainer/consumed_tokens": int(state.consumed_tokens),
                   "data/epoch": int(state.data_epoch),
                   "data/sample_offset": int(state.data_sample_offset),
                   "data/shuffle_seed": state.data_shuffle_seed}
            row.update({f"{prefix}/{k}": float(v) for k, v in metrics.items()})
        else:
            row = rec.wandb_payload()
        self._run.log(row)

    def history_state(self):
        return self.history.state_dict()

    def flush(self) -> None:
        self.history.flush()

    def update_summary(self, values: Mapping[str, Any]) -> None:
        update = getattr(getattr(self._run, "summary", None), "update", None)
        if values and callable(update):
            update(dict(values))

    def finish(self) -> None:
        run, self._run = self._run, None
        try:
            done = getattr(run, "finish", None)
            if callable(done):
                done()
        finally:
            self.history.close()

    def _module(self):
        if self._wandb is None:
            try:
                self._wandb = importlib.import_module("wandb")
            except ImportError as e:
                raise ImportError("W&B logging is enabled but the `wandb` package is not "
                                  "installed") from e
        return self._wandb
