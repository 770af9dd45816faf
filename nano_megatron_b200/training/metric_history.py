"""The run's metric timeline: ``metrics.jsonl``, one JSON object per train or validation
event, replayed into the next run on resume.

Line format (version 1; the reference's, so either framework reads the other's files)::

    {"version": 1, "sequence": n, "step": s, "recorded_at": unix_time, "prefix": "train",
     "metrics": {name: value}, "trainer": {"consumed_samples", "consumed_tokens"},
     "data": {"epoch", "sample_offset", "shuffle_seed"}}

Keys are sorted and the line is strict JSON: a non-finite metric is written as one of the
strings ``"NaN"``, ``"Infinity"``, ``"-Infinity"``. ``sequence`` increases by one per event
over the whole life of a run, across resumes; ``step`` never decreases.

Resume. A checkpoint stores ``(last_sequence, last_step)`` of the timeline at the moment
it was saved. The new run reads the old file up to the checkpoint's step, checks that its
last event is exactly that pair (otherwise the file and the checkpoint tell different
stories and the run stops), writes those events into its own new file and continues the
sequence from there. Events the old run logged after the checkpoint are left out, so the
new timeline has no gap and no duplicate. A crash can leave a last line without its
newline; the reader drops such a line with a warning, any other bad line is an error.
"""

from __future__ import annotations

import json
import math
import time
import warnings
from collections.abc import Iterator, Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

METRIC_HISTORY_VERSION = 1
_TEXT_OF = {math.inf: "Infinity", -math.inf: "-Infinity"}
_VALUE_OF = {"NaN": math.nan, "Infinity": math.inf, "-Infinity": -math.inf}


def _count(what: str, v: Any) -> int:
    if type(v) is not int or v < 0:
        raise ValueError(f"{what}: expected an int >= 0, got {v!r}")
    return v


def _maybe_count(what: str, v: Any) -> int | None:
    return None if v is None else _count(what, v)


def _number(name: str, v: Any) -> float:
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        raise TypeError(f"metric {name!r} is {v!r}, not a number")
    return float(v)


def _to_json_value(x: float):
    if math.isnan(x):
        return "NaN"
    return _TEXT_OF.get(x, x)


def _from_json_value(name: str, v: Any) -> float:
    if not isinstance(v, str):
        return _number(name, v)
    if v not in _VALUE_OF:
        raise ValueError(f"metric {name!r}: {v!r} is not NaN/Infinity/-Infinity")
    return _VALUE_OF[v]


def _prefix(v: Any) -> str:
    if not isinstance(v, str) or not v.strip():
        raise ValueError(f"metric prefix must be a non-blank string, got {v!r}")
    return v.strip()


# record field <- (section of the JSON object or None for the top level, key, checker)
_PROGRESS = (
    ("consumed_samples", "trainer", "consumed_samples", _count),
    ("consumed_tokens", "trainer", "consumed_tokens", _count),
    ("data_epoch", "data", "epoch", _count),
    ("data_sample_offset", "data", "sample_offset", _count),
    ("data_shuffle_seed", "data", "shuffle_seed", _maybe_count),
)


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
        """A new event from the trainer state (``TrainerState``-like) at this moment."""
        progress = {
            "consumed_samples": int(state.consumed_samples),
            "consumed_tokens": int(state.consumed_tokens),
            "data_epoch": int(state.data_epoch),
            "data_sample_offset": int(state.data_sample_offset),
            "data_shuffle_seed": state.data_shuffle_seed,
        }
        checked = {f: check(f, progress[f]) for f, _, _, check in _PROGRESS}
        return cls(sequence=_count("sequence", sequence), step=_count("step", int(state.step)),
                   recorded_at=time.time(), prefix=_prefix(prefix),
                   metrics={str(k): _number(str(k), v) for k, v in metrics.items()}, **checked)

    @classmethod
    def from_dict(cls, obj: Mapping[str, Any]) -> "MetricHistoryRecord":
        if obj.get("version") != METRIC_HISTORY_VERSION:
            raise ValueError(f"metric line has version {obj.get('version')!r}; this reader "
                             f"knows version {METRIC_HISTORY_VERSION}")
        sections = {}
        for name in ("metrics", "trainer", "data"):
            sec = obj.get(name)
            if not isinstance(sec, Mapping):
                raise TypeError(f"metric line field {name!r} must be an object")
            sections[name] = sec
        at = obj.get("recorded_at")
        if isinstance(at, bool) or not isinstance(at, (int, float)) or not \
                (math.isfinite(at) and at >= 0):
            raise ValueError(f"recorded_at {at!r} is not a finite time >= 0")
        progress = {f: check(f, sections[sec].get(key)) for f, sec, key, check in _PROGRESS}
        return cls(sequence=_count("sequence", obj.get("sequence")),
                   step=_count("step", obj.get("step")), recorded_at=float(at),
                   prefix=_prefix(obj.get("prefix")),
                   metrics={str(k): _from_json_value(str(k), v)
                            for k, v in sections["metrics"].items()}, **progress)

    def to_dict(self) -> dict[str, Any]:
        obj: dict[str, Any] = {
            "version": METRIC_HISTORY_VERSION, "sequence": self.sequence, "step": self.step,
            "recorded_at": self.recorded_at, "prefix": self.prefix,
            "metrics": {k: _to_json_value(v) for k, v in self.metrics.items()},
            "trainer": {}, "data": {}}
        for f, sec, key, _ in _PROGRESS:
            obj[sec][key] = getattr(self, f)
        return obj

    def to_json_line(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True, separators=(",", ":"),
                          ensure_ascii=False, allow_nan=False)

    def wandb_payload(self) -> dict[str, Any]:
        """Flat W&B row: ``trainer/*`` and ``data/*`` progress plus ``<prefix>/<metric>``."""
        row: dict[str, Any] = {"trainer/step": self.step}
        for f, sec, key, _ in _PROGRESS:
            row[f"{sec}/{key}"] = getattr(self, f)
        row.update({f"{self.prefix}/{k}": v for k, v in self.metrics.items()})
        return row


def _numbered_lines(path: Path) -> Iterator[tuple[int, str, bool]]:
    """(line number, text, whether it is the file's last line without a newline)."""
    with Path(path).open("r", encoding="utf-8") as f:
        lines = f.readlines()
    for i, line in enumerate(lines):
        yield i + 1, line, i == len(lines) - 1 and not line.endswith("\n")


def read_metric_history(path: Path, *, through_step: int | None = None
                        ) -> tuple[MetricHistoryRecord, ...]:
    """Every event of a timeline file (only those with ``step <= through_step`` if given),
    after checking the whole file: sequences strictly increasing, steps non-decreasing."""
    if through_step is not None:
        _count("through_step", through_step)
    kept: list[MetricHistoryRecord] = []
    prev: MetricHistoryRecord | None = None
    for n, line, unterminated in _numbered_lines(path):
        if not line.strip():
            continue
        try:
            obj = json.loads(line)
        except json.JSONDecodeError as e:
            if unterminated:
                warnings.warn(f"{path}:{n}: dropping a truncated last line (interrupted write)",
                              stacklevel=2)
                break
            raise ValueError(f"invalid metric history JSON at {path}:{n} ({e})") from e
        if not isinstance(obj, Mapping):
            raise TypeError(f"{path}:{n}: a metric line must be a JSON object")
        rec = MetricHistoryRecord.from_dict(obj)
        if prev is not None and rec.sequence <= prev.sequence:
            raise ValueError(f"{path}:{n}: sequences must increase ({prev.sequence} then "
                             f"{rec.sequence})")
        if prev is not None and rec.step < prev.step:
            raise ValueError(f"{path}:{n}: step went back from {prev.step} to {rec.step}")
        prev = rec
        if through_step is None or rec.step <= through_step:
            kept.append(rec)
    return tuple(kept)


class JsonlMetricHistory:
    """Writer of this run's timeline; on resume it first carries over the previous run's
    events up to the checkpoint (``start``), then ``append`` adds new ones."""

    def __init__(self, destination: Path | None, *, source: Path | None = None,
                 enabled: bool = True) -> None:
        self.destination = None if destination is None else Path(destination)
        self.source = None if source is None else Path(source)
        self.enabled = bool(enabled) and self.destination is not None
        self.replay_records: tuple[MetricHistoryRecord, ...] = ()
        self.source_missing = False
        self._out = None
        self._tail: MetricHistoryRecord | None = None     # last event written

    @property
    def _next_sequence(self) -> int:
        return 0 if self._tail is None else self._tail.sequence + 1

    def _previous_events(self, through_step: int | None) -> tuple[MetricHistoryRecord, ...]:
        if self.source is None:
            return ()
        if through_step is None:
            raise ValueError("resuming a metric timeline needs the checkpoint step")
        if not self.source.exists():
            self.source_missing = True
            warnings.warn(f"previous metric timeline {self.source} is missing; this run's "
                          "timeline (and its W&B child) starts without the earlier events",
                          stacklevel=3)
            return ()
        if self.source.resolve() == self.destination.resolve():
            raise ValueError(f"{self.source} is both the previous and the new timeline; they "
                             "must be distinct files")
        return read_metric_history(self.source, through_step=through_step)

    def start(self, *, through_step: int | None, expected_state: Mapping[str, Any] | None = None
              ) -> tuple[MetricHistoryRecord, ...]:
        """Open the new file (it must not exist yet) and write the carried-over events;
        returns them (for W&B replay). A second call returns the same events."""
        if not self.enabled:
            return ()
        if self._out is not None:
            return self.replay_records
        events = self._previous_events(through_step)
        if expected_state is not None:
            self._agree_with_checkpoint(events, expected_state)
        self.destination.parent.mkdir(parents=True, exist_ok=True)
        self._out = self.destination.open("x", encoding="utf-8", newline="\n")
        self._out.writelines(e.to_json_line() + "\n" for e in events)
        self._out.flush()
        self.replay_records = events
        self._tail = events[-1] if events else None
        return events

    def _agree_with_checkpoint(self, events, state: Mapping[str, Any]) -> None:
        if state.get("version") != METRIC_HISTORY_VERSION:
            raise ValueError(f"the checkpoint's metric-timeline entry has version "
                             f"{state.get('version')!r}, expected {METRIC_HISTORY_VERSION}")
        want = (_maybe_count("checkpoint last_sequence", state.get("last_sequence")),
                _maybe_count("checkpoint last_step", state.get("last_step")))
        if self.source_missing:
            return
        have = (events[-1].sequence, events[-1].step) if events else (None, None)
        if have != want:
            raise RuntimeError(f"metric history does not match the checkpoint: the checkpoint "
                               f"ends at (sequence, step) {want}, the file at {have}")

    def append(self, prefix: str, metrics: Mapping[str, float], *, state
               ) -> MetricHistoryRecord | None:
        if not self.enabled:
            return None
        if self._out is None:
            raise RuntimeError("call start() before appending metric events")
        rec = MetricHistoryRecord.capture(sequence=self._next_sequence, prefix=prefix,
                                          metrics=metrics, state=state)
        self._out.write(rec.to_json_line() + "\n")
        self._out.flush()
        self._tail = rec
        return rec

    def state_dict(self) -> dict | None:
        """The checkpoint's entry: where the timeline stands (None when disabled)."""
        if not self.enabled:
            return None
        tail = self._tail
        return {"version": METRIC_HISTORY_VERSION,
                "last_sequence": tail.sequence if tail else None,
                "last_step": tail.step if tail else None}

    def flush(self) -> None:
        if self._out is not None:
            self._out.flush()

    def close(self) -> None:
        out, self._out = self._out, None
        if out is not None:
            try:
                out.flush()
            finally:
                out.close()
