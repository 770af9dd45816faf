"""Every benchmark layout runs end to end on CPU ranks (gloo), at toy size.

``bench.py --config C --gpus N`` builds its run config from ``WORKLOADS``; here the same
config (same parallel layout, schedule, data-parallel mode, context-parallel backend and
activation checkpointing) is shrunk to a toy model and trained for two steps on N gloo
ranks. Loss and gradient norm must be finite and identical on every rank that reports
them, and the loss must start near ln(V). Numerical equivalence of the individual
layouts with a single-rank run is covered by the parallel-equivalence tests.
"""

from __future__ import annotations

import importlib.util
import math
from pathlib import Path

import pytest
import torch

from dist_utils import run_ranks

ROOT = Path(__file__).parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("nmb_bench_layouts", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _toy(d: dict) -> dict:
    """Shrink a benchmark config to toy size, keeping every layout-relevant field."""
    m = d["model"]
    gqa = m["heads"] // (m.get("kv_heads") or m["heads"])
    heads = 16                  # head dim 8; kv heads stay divisible by TP (up to 4)
    d["model"] = dict(m, layers=4, hidden_size=128, ffn_hidden_size=96, heads=heads,
                      kv_heads=heads // gqa, seq_length=64, vocab_size=256)
    d["distributed"] = {"backend": "gloo", "device": "cpu", "timeout_minutes": 2}
    d["precision"] = {"params": "float32", "compute": "float32", "grad_reduce": "float32"}
    d["data_parallel"]["bucket_bytes"] = 1 << 14
    tr = d["training"]
    dp = d["parallel"]["data"]
    pp = d["parallel"]["pipeline"]
    tr["micro_batch_size"] = 1
    tr["gradient_accumulation_steps"] = max(2, pp) * (2 if pp > 1 else 1)
    tr["max_steps"] = 10
    d["lr_scheduler"].update(decay_steps=10)
    d["global_rows"] = tr["micro_batch_size"] * tr["gradient_accumulation_steps"] * dp
    return d


CASES = []
for _name, _w in _bench().WORKLOADS.items():
    for _n in sorted(_w["layouts"]):
        if _n > 1:
            CASES.append((_name, _n))


def _rank(rank, world, name):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = _toy(_bench().make_config_dict(world, 10, name))
    rows = d.pop("global_rows")
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    dp = comps.parallel.dp.size
    g = torch.Generator().manual_seed(100 + comps.parallel.coordinate.dp)
    losses = []
    for _ in range(2):
        ids = torch.randint(0, 256, (rows // dp, 65), generator=g)
        out = tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
                            if tr.batch_router.is_source else None)
        loss = float(out["loss_sum"]) / max(float(out["token_count"]), 1.0)
        gn = float(out["grad_norm"])
        assert math.isfinite(loss) and math.isfinite(gn), (name, rank, loss, gn)
        losses.append((loss, gn))
    # every rank reports the same (globally reduced) loss and gradient norm
    box = [None] * world
    torch.distributed.all_gather_object(box, losses)
    for other in box:
        for (l0, g0), (l1, g1) in zip(losses, other):
            assert l1 == pytest.approx(l0, rel=1e-6) and g1 == pytest.approx(g0, rel=1e-5)
    assert abs(losses[0][0] - math.log(256)) < 0.5, losses


@pytest.mark.distributed
@pytest.mark.parametrize("name,world", CASES, ids=[f"{n}-{w}" for n, w in CASES])
def test_bench_layout_trains_on_gloo(name, world):
    run_ranks(world, _rank, name, timeout=600)
