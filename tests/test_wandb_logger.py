"""The optional W&B logger, driven by a fake ``wandb`` module (no network, no package).

Mirrors the reference's logger unit tests (tests/unit/test_wandb_logger.py:43-259): only
the primary rank of an enabled config ever calls ``wandb.init``; a fresh run may resume
its own id, a resumed run never continues the checkpoint's W&B run but starts a logical
child that replays the checkpoint's metric prefix and records its lineage; the local
``metrics.jsonl`` timeline is written whether W&B is enabled or not.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from nano_megatron_b200.config.schema import WandbConfig
from nano_megatron_b200.training.metric_history import read_metric_history
from nano_megatron_b200.training.wandb_logger import WandbLogger


class _Run:
    def __init__(self, **kw):
        self.kw, self.id = kw, kw.get("id")
        self.logged: list = []
        self.summary = type("Summary", (dict,), {"update": dict.update})()
        self.finished = False

    def log(self, payload):
        self.logged.append(dict(payload))

    def finish(self):
        self.finished = True


class _Wandb:
    def __init__(self):
        self.runs: list = []
        self.defined: list = []
        self.util = SimpleNamespace(generate_id=lambda: f"gen{len(self.runs)}")

    def init(self, **kw):
        self.runs.append(_Run(**kw))
        return self.runs[-1]

    def define_metric(self, *a, **kw):
        self.defined.append((a, kw))


def _state(step):
    return SimpleNamespace(step=step, consumed_samples=2 * step, consumed_tokens=32 * step,
                           data_epoch=0, data_sample_offset=2 * step, data_shuffle_seed=None)


def _logger(tmp_path, name, fake, *, primary=True, source=None, **cfg):
    c = WandbConfig(**{"enabled": True, "mode": "offline", **cfg})
    return WandbLogger(c, run_config={"model": {"layers": 2}}, is_primary=primary,
                       wandb_module=fake, metrics_path=tmp_path / name / "metrics.jsonl",
                       resume_metrics_path=source)


@pytest.mark.parametrize("enabled,primary", [(False, True), (True, False)])
def test_disabled_or_non_primary_logger_never_initializes_wandb(tmp_path, enabled, primary):
    fake = _Wandb()
    lg = _logger(tmp_path, "r", fake, primary=primary, enabled=enabled)
    assert lg.start() is None
    lg.log("train", {"loss": 1.0}, state=_state(1))
    lg.finish()
    assert fake.runs == []
    # the local timeline belongs to the primary rank only
    assert (tmp_path / "r" / "metrics.jsonl").exists() == primary


def test_disabled_wandb_still_writes_the_metric_timeline(tmp_path):
    lg = _logger(tmp_path, "r", _Wandb(), enabled=False)
    lg.start()
    for s in (1, 2):
        lg.log("train", {"loss": 3.0 - s}, state=_state(s))
    lg.finish()
    assert [r.step for r in read_metric_history(tmp_path / "r" / "metrics.jsonl")] == [1, 2]


def test_fresh_run_uses_the_configured_id_and_may_resume_it(tmp_path):
    fake = _Wandb()
    lg = _logger(tmp_path, "r", fake, run_id="mine")
    assert lg.start() == "mine"
    run = fake.runs[0]
    assert run.kw["resume"] == "allow" and run.kw["id"] == "mine"
    assert run.kw["config"] == {"model": {"layers": 2}}
    lg.log("train", {"loss": 2.0}, state=_state(1))
    assert run.logged[-1]["train/loss"] == 2.0 and run.logged[-1]["trainer/step"] == 1
    assert (("train/*",), {"step_metric": "trainer/step"}) in fake.defined
    lg.finish()
    assert run.finished


def test_resume_replays_the_prefix_into_a_logical_child_and_records_lineage(tmp_path):
    fake = _Wandb()
    first = _logger(tmp_path, "r1", fake)
    first.start()
    for s in (1, 2, 3):
        first.log("train", {"loss": 5.0 - s}, state=_state(s))
    first.finish()
    src_id = fake.runs[0].id
    # the checkpoint was taken at step 2, after the timeline's second record
    child = _logger(tmp_path, "r2", fake, source=tmp_path / "r1" / "metrics.jsonl")
    rid = child.start(checkpoint_run_id=src_id, checkpoint_step=2,
                      checkpoint_metrics_state={"version": 1, "last_sequence": 1,
                                                "last_step": 2})
    run = fake.runs[1]
    assert rid != src_id and run.kw["resume"] == "never"
    assert [p["trainer/step"] for p in run.logged] == [1, 2]
    assert run.summary["wandb/forked_from_run_id"] == src_id
    assert run.summary["wandb/forked_from_step"] == 2
    assert run.summary["wandb/history_replayed_records"] == 2
    child.log("train", {"loss": 1.5}, state=_state(3))
    child.finish()
    assert [r.sequence for r in read_metric_history(tmp_path / "r2" / "metrics.jsonl")] == \
        [0, 1, 2]


def test_fork_replaces_a_configured_id_equal_to_the_source_run(tmp_path):
    fake = _Wandb()
    lg = _logger(tmp_path, "r", fake, run_id="src")
    rid = lg.start(checkpoint_run_id="src", checkpoint_step=0)
    assert rid != "src" and fake.runs[0].kw["resume"] == "never"


def test_fork_uses_a_new_configured_id(tmp_path):
    fake = _Wandb()
    lg = _logger(tmp_path, "r", fake, run_id="child")
    assert lg.start(checkpoint_run_id="src", checkpoint_step=0) == "child"


def test_fork_requires_the_checkpoint_step(tmp_path):
    lg = _logger(tmp_path, "r", _Wandb())
    with pytest.raises(ValueError, match="checkpoint_step"):
        lg.start(checkpoint_run_id="src")
    with pytest.raises(ValueError, match="non-negative"):
        lg.start(checkpoint_step=-1)
