"""The versioned ``metrics.jsonl`` timeline: encoding, resume replay and damaged files.

Mirrors the reference's metric-history unit tests (tests/unit/test_metric_history.py:24-152):
non-finite metrics round-trip through strict JSON; a resumed run copies exactly the
checkpoint's prefix of the previous timeline and continues its sequence numbers; a missing
previous timeline warns and starts empty; a timeline that disagrees with the checkpoint is
rejected; a final line cut off mid-write is dropped, any other invalid line is an error.
"""

from __future__ import annotations

import json
import math
from types import SimpleNamespace

import pytest

from nano_megatron_b200.training.metric_history import (JsonlMetricHistory,
                                                        MetricHistoryRecord,
                                                        read_metric_history)


def _state(step: int):
    return SimpleNamespace(step=step, consumed_samples=4 * step, consumed_tokens=256 * step,
                           data_epoch=0, data_sample_offset=4 * step, data_shuffle_seed=7)


def _write_run(path, steps):
    h = JsonlMetricHistory(path)
    h.start(through_step=None)
    for s in steps:
        h.append("train", {"loss": 10.0 - s, "lr": 1e-3}, state=_state(s))
        if s % 2 == 0:
            h.append("validation", {"loss": 9.5 - s}, state=_state(s))
    sd = h.state_dict()
    h.close()
    return sd


def test_nonfinite_metrics_round_trip_as_strict_json(tmp_path):
    p = tmp_path / "metrics.jsonl"
    h = JsonlMetricHistory(p)
    h.start(through_step=None)
    h.append("train", {"loss": float("nan"), "grad_norm": float("inf"),
                       "delta": float("-inf"), "lr": 3e-4}, state=_state(1))
    h.close()
    line = p.read_text().strip()
    json.loads(line, parse_constant=lambda c: pytest.fail(f"non-standard JSON token {c}"))
    (r,) = read_metric_history(p)
    assert math.isnan(r.metrics["loss"])
    assert r.metrics["grad_norm"] == float("inf") and r.metrics["delta"] == float("-inf")
    assert r.metrics["lr"] == 3e-4 and r.step == 1 and r.prefix == "train"
    assert r.consumed_tokens == 256 and r.data_shuffle_seed == 7
    assert MetricHistoryRecord.from_dict(json.loads(line)) == r


def test_resume_copies_only_the_checkpoint_prefix_and_continues_the_sequence(tmp_path):
    old = tmp_path / "run1" / "metrics.jsonl"
    _write_run(old, range(1, 7))
    # the checkpoint was taken at step 4: the timeline's state at that point
    upto = [r for r in read_metric_history(old) if r.step <= 4]
    expected = {"version": 1, "last_sequence": upto[-1].sequence, "last_step": 4}
    new = tmp_path / "run2" / "metrics.jsonl"
    h = JsonlMetricHistory(new, source=old)
    replay = h.start(through_step=4, expected_state=expected)
    assert [r.step for r in replay] == [r.step for r in upto]
    rec = h.append("train", {"loss": 5.0}, state=_state(5))
    assert rec.sequence == upto[-1].sequence + 1
    h.close()
    got = read_metric_history(new)
    assert [r.sequence for r in got] == list(range(len(upto) + 1))
    assert [r.step for r in got][-1] == 5
    # the previous run's file is left as it was
    assert len(read_metric_history(old)) > len(upto)


def test_missing_previous_timeline_warns_and_starts_empty(tmp_path):
    h = JsonlMetricHistory(tmp_path / "new.jsonl", source=tmp_path / "absent.jsonl")
    with pytest.warns(UserWarning, match="missing"):
        replay = h.start(through_step=3, expected_state={"version": 1, "last_sequence": 5,
                                                          "last_step": 3})
    assert replay == () and h.source_missing
    assert h.append("train", {"loss": 1.0}, state=_state(4)).sequence == 0
    h.close()


def test_missing_previous_timeline_still_checks_the_checkpoint_version(tmp_path):
    h = JsonlMetricHistory(tmp_path / "new.jsonl", source=tmp_path / "absent.jsonl")
    with pytest.warns(UserWarning), pytest.raises(ValueError, match="version"):
        h.start(through_step=3, expected_state={"version": 2, "last_sequence": 5,
                                                "last_step": 3})


def test_timeline_that_disagrees_with_the_checkpoint_is_rejected(tmp_path):
    old = tmp_path / "old.jsonl"
    _write_run(old, range(1, 5))
    h = JsonlMetricHistory(tmp_path / "new.jsonl", source=old)
    with pytest.raises(RuntimeError, match="does not match the checkpoint"):
        h.start(through_step=4, expected_state={"version": 1, "last_sequence": 99,
                                                "last_step": 4})


def test_resume_requires_a_checkpoint_step_and_distinct_files(tmp_path):
    old = tmp_path / "old.jsonl"
    _write_run(old, [1])
    with pytest.raises(ValueError, match="checkpoint step"):
        JsonlMetricHistory(tmp_path / "n.jsonl", source=old).start(through_step=None)
    with pytest.raises(ValueError, match="distinct"):
        JsonlMetricHistory(old, source=old).start(through_step=1)


def test_reader_drops_only_a_truncated_final_line(tmp_path):
    p = tmp_path / "m.jsonl"
    _write_run(p, [1, 2])
    n = len(read_metric_history(p))
    text = p.read_text()
    p.write_text(text + text.splitlines()[0][:25])           # crash mid-write: no newline
    with pytest.warns(UserWarning, match="truncated"):
        assert len(read_metric_history(p)) == n


def test_reader_rejects_an_invalid_complete_final_line(tmp_path):
    p = tmp_path / "m.jsonl"
    _write_run(p, [1, 2])
    p.write_text(p.read_text() + "{not json}\n")
    with pytest.raises(ValueError, match="invalid metric history JSON"):
        read_metric_history(p)


def test_reader_rejects_sequences_that_do_not_increase(tmp_path):
    p = tmp_path / "m.jsonl"
    _write_run(p, [1, 2])
    lines = p.read_text().splitlines()
    p.write_text("\n".join([lines[0], lines[0]]) + "\n")
    with pytest.raises(ValueError, match="sequences must increase"):
        read_metric_history(p)


def test_disabled_history_writes_nothing(tmp_path):
    h = JsonlMetricHistory(tmp_path / "m.jsonl", enabled=False)
    assert h.start(through_step=None) == ()
    assert h.append("train", {"loss": 1.0}, state=_state(1)) is None
    assert h.state_dict() is None
    assert not (tmp_path / "m.jsonl").exists()
