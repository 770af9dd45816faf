"""bench.py's model-FLOPs annotation: the 311M GPT's training FLOPs per token and the
fraction of the measured sustained bf16 rate that a throughput implies."""

import importlib.util
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("nmb_bench_roofline", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_311m_flops_per_token():
    b = _bench()
    m = b.WORKLOADS["311m"]["model"]
    params = 24 * (1024 * 3072 + 1024 * 1024 + 1024 * 2 * 2736 + 2736 * 1024) + 8192 * 1024
    assert params == pytest.approx(310.8e6, rel=1e-3)            # the "311M" of the name
    assert b.model_flops_per_token(m) == 6 * params + 6 * 24 * 1024 * 512


def test_roofline_fraction_uses_the_measured_sustained_peak():
    b = _bench()
    w = b.WORKLOADS["311m"]
    out = b.roofline(w, 100_000.0, 2)
    assert out["model_tflops_per_gpu"] == pytest.approx(
        b.model_flops_per_token(w["model"]) * 50_000 / 1e12)
    peaks = ROOT / "MEASURED_PEAKS.json"
    if peaks.exists():
        sustained = json.loads(peaks.read_text())["bf16_tflops_sustained"]
        assert out["frac_of_measured_bf16_sustained"] == pytest.approx(
            out["model_tflops_per_gpu"] / sustained)
