"""Optional, primary-rank-only Weights & Biases telemetry on top of the local metric history.

``wandb`` is imported only when enabled. A resumed run never continues the
checkpoint's W&B run: it starts a fresh run (``resume="never"``), replays the
checkpoint-consistent metric prefix into it and records the lineage
(``wandb/forked_from_*``) in the summary -- the reference's policy
(src/nano_megatron/training/wandb_logger.py:26-222).
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
    if is_dataclass(v) and not isinstance(v, type):
        return {f.name: plain_config(getattr(v, f.name)) for f in fields(v)}
    if isinstance(v, Mapping):
        return {str(k): plain_config(x) for k, x in v.items()}
    if isinstance(v, (tuple, list)):
        return [plain_config(x) for x in v]
    if isinstance(v, (Enum, Path)):
        return str(getattr(v, "value", v))
    return v


class WandbLogger:
    def __init__(self, config, *, run_config, is_primary: bool, wandb_module=None,
                 metrics_path: Path | None = None, resume_metrics_path: Path | None = None) -> None:
        self.config = config
        self.run_config = run_config
        self.enabled = bool(config is not None and config.enabled and
                            config.mode != "disabled" and is_primary)
        self._wandb = wandb_module
        self._run = None
        self.run_id: str | None = None
        self.history = JsonlMetricHistory(metrics_path, source=resume_metrics_path,
                                          enabled=is_primary)

    def start(self, *, checkpoint_run_id: str | None = None, checkpoint_step: int | None = None,
              checkpoint_metrics_state: Mapping[str, Any] | None = None, model=None
              ) -> str | None:
        if self._run is not None:
            return self.run_id
        restore = checkpoint_step is not None
        if checkpoint_run_id is not None and not restore:
            raise ValueError("checkpoint_run_id requires checkpoint_step")
        if restore and (isinstance(checkpoint_step, bool) or not isinstance(checkpoint_step, int)
                        or checkpoint_step < 0):
            raise ValueError("checkpoint_step must be a non-negative integer on restore")
        replay = self.history.start(through_step=checkpoint_step,
                                    expected_state=checkpoint_metrics_state)
        if not self.enabled:
            return None
        mod = self._module()
        want = self.config.run_id
        if not restore:
            rid = want or self._new_id(mod)
        else:
            rid = want if want is not None and want != checkpoint_run_id else self._new_id(mod)
            if rid == checkpoint_run_id:
                rid = uuid.uuid4().hex
        opts = {"project": self.config.project, "entity": self.config.entity,
                "name": self.config.name, "group": self.config.group,
                "tags": list(self.config.tags), "mode": self.config.mode,
                "dir": None if self.config.directory is None else str(self.config.directory),
                "id": rid, "config": plain_config(self.run_config),
                "resume": "never" if restore else "allow"}
        self._run = mod.init(**{k: v for k, v in opts.items() if v is not None})
        if self._run is None:
            raise RuntimeError("wandb.init() returned no run")
        got = getattr(self._run, "id", rid)
        if not isinstance(got, str) or not got:
            raise RuntimeError("W&B run must expose a non-empty string id")
        self.run_id = got
        define = getattr(mod, "define_metric", None)
        if callable(define):
            define("trainer/step")
            define("train/*", step_metric="trainer/step")
            define("validation/*", step_metric="trainer/step")
        for r in replay:
            self._run.log(r.wandb_payload())
        if restore:
            lineage = {"wandb/logical_fork": True, "wandb/forked_from_step": checkpoint_step,
                       "wandb/history_replayed_records": len(replay)}
            if checkpoint_run_id is not None:
                lineage["wandb/forked_from_run_id"] = checkpoint_run_id
            self.update_summary(lineage)
        if self.history.destination is not None:
            self.update_summary({"metrics/history_path": str(self.history.destination)})
        if model is not None:
            ps = list(model.parameters())
            self.update_summary({"model/parameters": sum(p.numel() for p in ps),
                                 "model/trainable_parameters":
                                     sum(p.numel() for p in ps if p.requires_grad)})
        return self.run_id

    def log(self, prefix: str, metrics: Mapping[str, float], *, state) -> None:
        r = self.history.append(prefix, metrics, state=state)
        if self._run is None:
            return
        if r is not None:
            payload = r.wandb_payload()
        else:
            payload = {"trainer/step": int(state.step),
                       "trainer/consumed_samples": int(state.consumed_samples),
                       "trainer/consumed_tokens": int(state.consumed_tokens),
                       "data/epoch": int(state.data_epoch),
                       "data/sample_offset": int(state.data_sample_offset),
                       "data/shuffle_seed": state.data_shuffle_seed}
            payload.update({f"{prefix}/{k}": float(v) for k, v in metrics.items()})
        self._run.log(payload)

    def history_state(self):
        return self.history.state_dict()

    def flush(self) -> None:
        self.history.flush()

    def update_summary(self, values: Mapping[str, Any]) -> None:
        upd = getattr(getattr(self._run, "summary", None), "update", None)
        if callable(upd):
            upd(dict(values))

    def finish(self) -> None:
        try:
            fin = getattr(self._run, "finish", None)
            if callable(fin):
                fin()
        finally:
            self._run = None
            self.history.close()

    def _module(self):
        if self._wandb is None:
            try:
                self._wandb = importlib.import_module("wandb")
            except ImportError as e:
                raise ImportError("wandb.enabled=true requires the optional tracking dependency "
                                  "`wandb`") from e
        return self._wandb

    @staticmethod
    def _new_id(mod) -> str:
        gen = getattr(getattr(mod, "util", None), "generate_id", None)
        if callable(gen):
            v = gen()
            if isinstance(v, str) and v:
                return v
        return uuid.uuid4().hex
