"""Deterministic kernel mode, host side: the config field, the process-wide switch, and the
portable run config (the field is dropped at its default so the reference's strict loader
still reads our manifests). The kernels themselves are covered by
``test_deterministic_gpu.py``."""

import pytest

from nano_megatron_b200.checkpoint.manager import portable_run_config
from nano_megatron_b200.config import config_from_dict
from nano_megatron_b200.ops import _ext
from nano_megatron_b200.ops import deterministic as det


def test_config_field_defaults_off_and_must_be_boolean():
    assert config_from_dict({}).kernels.deterministic is False
    assert config_from_dict({"kernels": {"deterministic": True}}).kernels.deterministic is True
    with pytest.raises((TypeError, ValueError)):
        config_from_dict({"kernels": {"deterministic": "yes"}})


def test_portable_run_config_drops_the_field_only_at_its_default():
    off = portable_run_config(config_from_dict({}))
    assert "deterministic" not in off["kernels"]
    on = portable_run_config(config_from_dict({"kernels": {"deterministic": True}}))
    assert on["kernels"]["deterministic"] is True


def test_switch_context_and_configure(monkeypatch):
    monkeypatch.delenv("NMB_DETERMINISTIC", raising=False)
    det.set_deterministic(False)
    with det.deterministic():
        assert det.is_deterministic()
        with det.deterministic(False):
            assert not det.is_deterministic()
        assert det.is_deterministic()
    assert not det.is_deterministic()
    det.configure(True)
    assert det.is_deterministic()
    det.configure(False)
    assert not det.is_deterministic()
    monkeypatch.setenv("NMB_DETERMINISTIC", "1")
    det.configure(False)  # the environment asks for it
    assert det.is_deterministic()
    monkeypatch.setenv("NMB_DETERMINISTIC", "0")
    det.configure(False)
    assert not det.is_deterministic()


@pytest.mark.skipif(not _ext.available(), reason="kernel library not built")
def test_switch_reaches_the_kernel_library_flag():
    try:
        det.set_deterministic(True)
        assert _ext.lib().get_deterministic()
    finally:
        det.set_deterministic(False)
    assert not _ext.lib().get_deterministic()


def test_building_components_applies_the_config(monkeypatch):
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training.engine import build_training_components

    monkeypatch.delenv("NMB_DETERMINISTIC", raising=False)
    model = {"layers": 1, "hidden_size": 64, "ffn_hidden_size": 128, "heads": 2,
             "kv_heads": 2, "seq_length": 16, "vocab_size": 128}
    try:
        for flag in (True, False):
            cfg = config_from_dict({"model": model, "kernels": {"deterministic": flag},
                                    "distributed": {"device": "cpu", "backend": "gloo"}})
            build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
            assert det.is_deterministic() is flag
    finally:
        det.set_deterministic(False)
