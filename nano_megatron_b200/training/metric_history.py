"""Versioned JSONL metric timeline (``metrics.jsonl``) with checkpoint-consistent replay.

Each line is one train or validation event: ``version`` (1), a strictly
increasing ``sequence``, the trainer ``step``, ``recorded_at``, a ``prefix``
(``train``/``validation``), the metrics (non-finite values written as the
strings ``NaN``/``Infinity``/``-Infinity`` so every line is strict JSON), and
the trainer and data progress. On resume the previous run's timeline is read
up to the checkpoint step, checked against the (last sequence, last step)
stored in the checkpoint, and copied into the new run's file before new events
are appended. Same record schema as the reference
(src/nano_megatron/training/metric_history.py:11-395).
"""

from __future__ import annotations

import json
import math
import time
import warnings
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

METRIC_HISTORY_VERSION = 1
_SPECIAL = {"NaN": float("nan"), "Infinity": float("inf"), "-Infinity": float("-inf")}


def _nonneg(name: str, v: Any) -> int:
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise ValueError(f"{name} must be a non-negative integer")
    return v


def _opt_nonneg(name: str, v: Any) -> int | None:
    return None if v is None else _nonneg(name, v)


def _num(name: str, v: Any) -> float:
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        raise TypeError(f"metric {name!r} must be numeric")
    return float(v)


def _enc(v: float):
    if math.isnan(v):
        return "NaN"
    if math.isinf(v):
        return "Infinity" if v > 0 else "-Infinity"
    return v


def _dec(name: str, v: Any) -> float:
    if isinstance(v, str):
        if v not in _SPECIAL:
            raise ValueError(f"metric {name!r} has an invalid string value {v!r}")
        return _SPECIAL[v]
    return _num(name, v)


@dataclass(frozen=True, slots=True)
class MetricHistoryRecord:
    sequence: int
    step: int
    recorded_at: float
    prefix: str
    metrics: dict
    consumed_samples: int
    consumed_tokens: int
    data_epoch: int
    data_sample_offset: int
    data_shuffle_seed: int | None

    @classmethod
    def capture(cls, *, sequence: int, prefix: str, metrics: Mapping[str, float], state
                ) -> "MetricHistoryRecord":
        if not isinstance(prefix, str) or not prefix.strip():
            raise ValueError("metric prefix must be a non-empty string")
        return cls(_nonneg("metric sequence", sequence), _nonneg("metric step", int(state.step)),
                   time.time(), prefix.strip(),
                   {str(k): _num(str(k), v) for k, v in metrics.items()},
                   _nonneg("consumed_samples", int(state.consumed_samples)),
                   _nonneg("consumed_tokens", int(state.consumed_tokens)),
                   _nonneg("data_epoch", int(state.data_epoch)),
                   _nonneg("data_sample_offset", int(state.data_sample_offset)),
                   _opt_nonneg("data_shuffle_seed", state.data_shuffle_seed))

    @classmethod
    def from_dict(cls, v: Mapping[str, Any]) -> "MetricHistoryRecord":
        if v.get("version") != METRIC_HISTORY_VERSION:
            raise ValueError(f"unsupported metric history version {v.get('version')!r}; "
                             f"expected {METRIC_HISTORY_VERSION}")
        prefix = v.get("prefix")
        if not isinstance(prefix, str) or not prefix.strip():
            raise ValueError("metric history prefix must be a non-empty string")
        metrics, trainer, data = v.get("metrics"), v.get("trainer"), v.get("data")
        if not isinstance(metrics, Mapping):
            raise TypeError("metric history metrics must be a mapping")
        if not isinstance(trainer, Mapping) or not isinstance(data, Mapping):
            raise TypeError("metric history trainer and data state must be mappings")
        at = v.get("recorded_at")
        if isinstance(at, bool) or not isinstance(at, (int, float)) or \
                not math.isfinite(float(at)) or float(at) < 0:
            raise ValueError("metric history recorded_at must be a finite non-negative number")
        return cls(_nonneg("metric sequence", v.get("sequence")),
                   _nonneg("metric step", v.get("step")), float(at), prefix.strip(),
                   {str(k): _dec(str(k), x) for k, x in metrics.items()},
                   _nonneg("consumed_samples", trainer.get("consumed_samples")),
                   _nonneg("consumed_tokens", trainer.get("consumed_tokens")),
                   _nonneg("data_epoch", data.get("epoch")),
                   _nonneg("data_sample_offset", data.get("sample_offset")),
                   _opt_nonneg("data_shuffle_seed", data.get("shuffle_seed")))

    def to_dict(self) -> dict[str, Any]:
        return {"version": METRIC_HISTORY_VERSION, "sequence": self.sequence, "step": self.step,
                "recorded_at": self.recorded_at, "prefix": self.prefix,
                "metrics": {k: _enc(x) for k, x in self.metrics.items()},
                "trainer": {"consumed_samples": self.consumed_samples,
                            "consumed_tokens": self.consumed_tokens},
                "data": {"epoch": self.data_epoch, "sample_offset": self.data_sample_offset,
                         "shuffle_seed": self.data_shuffle_seed}}

    def to_json_line(self) -> str:
        return json.dumps(self.to_dict(), ensure_ascii=False, separators=(",", ":"),
                          sort_keys=True, allow_nan=False)

    def wandb_payload(self) -> dict[str, Any]:
        out = {"trainer/step": self.step, "trainer/consumed_samples": self.consumed_samples,
               "trainer/consumed_tokens": self.consumed_tokens, "data/epoch": self.data_epoch,
               "data/sample_offset": self.data_sample_offset,
               "data/shuffle_seed": self.data_shuffle_seed}
        out.update({f"{self.prefix}/{k}": x for k, x in self.metrics.items()})
        return out


def read_metric_history(path: Path, *, through_step: int | None = None
                        ) -> tuple[MetricHistoryRecord, ...]:
    """Validated records (sequences increasing, steps non-decreasing), optionally <= a step.

    A truncated last line (a crash mid-write) is dropped with a warning."""
    if through_step is not None:
        _nonneg("metric history cutoff step", through_step)
    lines = Path(path).read_text(encoding="utf-8").split("\n")
    out: list[MetricHistoryRecord] = []
    last_seq = last_step = -1
    for n, line in enumerate(lines, start=1):
        if not line.strip():
            continue
        try:
            v = json.loads(line)
        except json.JSONDecodeError as e:
            if n == len(lines):            # no trailing newline: the final line was cut off
                warnings.warn(f"ignoring truncated final metric history line {n} in {path}",
                              stacklevel=2)
                break
            raise ValueError(f"invalid metric history JSON at {path}:{n}: {e}") from e
        if not isinstance(v, Mapping):
            raise TypeError(f"metric history line {path}:{n} must be an object")
        r = MetricHistoryRecord.from_dict(v)
        if r.sequence <= last_seq:
            raise ValueError(f"metric history sequences must increase at {path}:{n}")
        if r.step < last_step:
            raise ValueError(f"metric history steps must not decrease at {path}:{n}")
        last_seq, last_step = r.sequence, r.step
        if through_step is None or r.step <= through_step:
            out.append(r)
    return tuple(out)


class JsonlMetricHistory:
    """Copy a checkpoint's metric prefix into this run's file, then append new events."""

    def __init__(self, destination: Path | None, *, source: Path | None = None,
                 enabled: bool = True) -> None:
        self.destination = None if destination is None else Path(destination)
        self.source = None if source is None else Path(source)
        self.enabled = bool(enabled and self.destination is not None)
        self._f = None
        self._next = 0
        self._last: MetricHistoryRecord | None = None
        self.replay_records: tuple[MetricHistoryRecord, ...] = ()
        self.source_missing = False

    def start(self, *, through_step: int | None, expected_state: Mapping[str, Any] | None = None
              ) -> tuple[MetricHistoryRecord, ...]:
        if not self.enabled:
            return ()
        if self._f is not None:
            return self.replay_records
        if self.source is not None and through_step is None:
            raise ValueError("resume metric history requires a checkpoint step")
        replay: tuple[MetricHistoryRecord, ...] = ()
        if self.source is not None:
            if self.source.exists():
                if self.source.resolve() == self.destination.resolve():
                    raise ValueError("source and destination metric histories must be distinct")
                replay = read_metric_history(self.source, through_step=through_step)
            else:
                self.source_missing = True
                warnings.warn(f"resume metric history is missing: {self.source}; the logical "
                              "W&B child will start without replayed metrics", stacklevel=2)
        self._check(replay, expected_state)
        self.destination.parent.mkdir(parents=True, exist_ok=True)
        self._f = self.destination.open("x", encoding="utf-8", newline="\n")
        for r in replay:
            self._f.write(r.to_json_line() + "\n")
        self._f.flush()
        self.replay_records = replay
        if replay:
            self._last, self._next = replay[-1], replay[-1].sequence + 1
        return replay

    def append(self, prefix: str, metrics: Mapping[str, float], *, state
               ) -> MetricHistoryRecord | None:
        if not self.enabled:
            return None
        if self._f is None:
            raise RuntimeError("metric history must be started before logging")
        r = MetricHistoryRecord.capture(sequence=self._next, prefix=prefix, metrics=metrics,
                                        state=state)
        self._f.write(r.to_json_line() + "\n")
        self._f.flush()
        self._next += 1
        self._last = r
        return r

    def state_dict(self) -> dict | None:
        if not self.enabled:
            return None
        return {"version": METRIC_HISTORY_VERSION,
                "last_sequence": None if self._last is None else self._last.sequence,
                "last_step": None if self._last is None else self._last.step}

    def flush(self) -> None:
        if self._f is not None:
            self._f.flush()

    def close(self) -> None:
        if self._f is not None:
            try:
                self._f.flush()
            finally:
                self._f.close()
                self._f = None

    def _check(self, replay, expected) -> None:
        if expected is None:
            return
        if expected.get("version") != METRIC_HISTORY_VERSION:
            raise ValueError(f"checkpoint metric history version {expected.get('version')!r} is "
                             f"unsupported; expected {METRIC_HISTORY_VERSION}")
        got = (replay[-1].sequence, replay[-1].step) if replay else (None, None)
        want = (_opt_nonneg("checkpoint metric history last_sequence",
                            expected.get("last_sequence")),
                _opt_nonneg("checkpoint metric history last_step", expected.get("last_step")))
        if not self.source_missing and got != want:
            raise RuntimeError(f"metric history does not match the checkpoint: expected "
                               f"sequence/step {want}, got {got}")
