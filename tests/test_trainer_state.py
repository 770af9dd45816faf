"""Trainer progress state: checkpoint round trip, validation of restored values, data binding.

Mirrors the reference's trainer-state unit tests (tests/unit/test_trainer_state.py:11-100):
the state survives a round trip; partial or invalid best-validation records are rejected;
a resumed trainer refuses data whose fingerprint differs from the checkpoint's and moves a
resumable loader to the checkpoint's position before the first batch.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from nano_megatron_b200.training.trainer import Trainer, TrainerState


def _full_state() -> TrainerState:
    return TrainerState(step=12, consumed_samples=96, consumed_tokens=96 * 128,
                        data_fingerprint="sha256:abc", data_epoch=1, data_shuffle_seed=5,
                        data_sample_offset=32, data_samples_per_epoch=64,
                        lr_scheduler={"completed_steps": 12}, wandb_run_id="run-1",
                        metrics_history={"version": 1, "last_sequence": 14, "last_step": 12},
                        best_validation_loss=2.5, best_validation_step=10,
                        best_validation_checkpoint="step_00000010")


def test_trainer_state_round_trip():
    st = _full_state()
    sd = st.state_dict()
    back = TrainerState()
    back.load_state_dict(sd)
    assert back.state_dict() == sd
    sd["lr_scheduler"]["completed_steps"] = 99          # the dict is a copy
    assert st.lr_scheduler == {"completed_steps": 12}


@pytest.mark.parametrize("bad", [
    {"best_validation_checkpoint": "step_1"},                         # no metrics
    {"best_validation_loss": 1.0},                                     # no step
    {"best_validation_loss": float("inf"), "best_validation_step": 1},
    {"best_validation_loss": -1.0, "best_validation_step": 1},
    {"best_validation_loss": 1.0, "best_validation_step": True},
    {"step": -1},
    {"data_shuffle_seed": -3},
    {"data_samples_per_epoch": 0},
    {"data_fingerprint": ""},
    {"wandb_run_id": ""},
    {"lr_scheduler": [1, 2]},
], ids=lambda d: ",".join(d))
def test_trainer_state_rejects_partial_or_invalid_values(bad):
    with pytest.raises(ValueError):
        TrainerState().load_state_dict(bad)


class _Loader:
    def __init__(self):
        self.restored = None

    def load_state_dict(self, st):
        self.restored = dict(st)

    def __iter__(self):
        return iter(())


def _host(state):
    return SimpleNamespace(state=state)


def test_bind_rejects_a_data_fingerprint_change_across_resume():
    host = _host(TrainerState(step=4, data_fingerprint="sha256:old"))
    with pytest.raises(RuntimeError, match="fingerprint"):
        Trainer.bind_data_iterator(host, _Loader(), data_fingerprint="sha256:new")
    Trainer.bind_data_iterator(host, _Loader(), data_fingerprint="sha256:old")
    assert host.state.data_fingerprint == "sha256:old"


def test_bind_moves_a_resumed_loader_to_the_checkpoint_position():
    host = _host(TrainerState(step=6, data_epoch=2, data_sample_offset=40,
                              data_shuffle_seed=9, data_samples_per_epoch=64))
    loader = _Loader()
    Trainer.bind_data_iterator(host, loader, data_fingerprint=None)
    assert loader.restored == {"epoch": 2, "sample_offset": 40, "shuffle_seed": 9,
                               "samples_per_epoch": 64}
    fresh = _Loader()
    Trainer.bind_data_iterator(_host(TrainerState()), fresh)
    assert fresh.restored is None                       # a fresh run starts at the beginning
