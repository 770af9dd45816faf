"""Training flows (CPU): W&B replay on resume with a fake wandb module, CLI resume under
ZeRO-2 + full activation checkpointing + offloads, async save while training continues,
a data-parallel expansion keeping the new replica's RNG with a warning, bitwise
reproducibility of multi-rank training (with dropout) across reruns, and the per-phase
step times in the fit log, and the overlapped DDP reducer's launch / wait order.
Reference counterparts: tests/integration/test_cli_resume.py:58-151,
tests/unit/test_data_parallel_buckets.py:55-282 (delayed all-reduce works),
tests/integration/test_wandb_training_flow.py, tests/unit/test_wandb_logger.py:12-41,
tests/distributed_cpu/test_checkpoint_rank_local.py:435, 605-700.
"""

from __future__ import annotations

import json
import warnings
from pathlib import Path

import pytest
import torch
import yaml

from dist_utils import run_ranks


class _FakeRun:
    def __init__(self, **kw):
        self.kw = kw
        self.id = kw.get("id", "run-x")
        self.logged: list = []
        self.summary = {}
        self.finished = False

    def log(self, payload):
        self.logged.append(dict(payload))

    def finish(self):
        self.finished = True


class _FakeWandb:
    def __init__(self):
        self.runs: list = []
        self.defined: list = []

    def init(self, **kw):
        run = _FakeRun(**kw)
        run.summary = type("S", (dict,), {"update": dict.update})()
        self.runs.append(run)
        return run

    def define_metric(self, *a, **kw):
        self.defined.append((a, kw))


def _base_cfg(tmp: Path, **over) -> dict:
    from nano_megatron_b200.config import TrainConfig
    from nano_megatron_b200.config.loader import config_to_dict

    d = config_to_dict(TrainConfig())
    d["distributed"].update(backend="gloo", device="cpu")
    d["model"].update(layers=2, hidden_size=32, ffn_hidden_size=64, heads=4, kv_heads=2,
                      seq_length=16, vocab_size=128)
    d["precision"].update(params="float32", compute="float32")
    d["training"].update(micro_batch_size=2, gradient_accumulation_steps=2, max_steps=4,
                         log_interval=1, seed=5)
    d["optimizer"].update(lr=1e-2)
    d["checkpoint"].update(directory=str(tmp / "runs"), save_interval=2, keep_last=4)
    for k, v in over.items():
        d[k].update(v)
    return d


def test_wandb_replay_and_fork_on_resume(tmp_path, monkeypatch):
    from nano_megatron_b200.cli import train as trcli
    from nano_megatron_b200.training import wandb_logger

    fake = _FakeWandb()
    monkeypatch.setattr(wandb_logger.importlib, "import_module",
                        lambda name: fake if name == "wandb" else __import__(name))
    cfg = tmp_path / "c.yaml"
    cfg.write_text(yaml.safe_dump(_base_cfg(tmp_path, wandb={"enabled": True,
                                                             "mode": "offline"})))
    trcli.run(cfg, max_steps=2, log=lambda *_: None)
    first = fake.runs[0]
    assert [p["trainer/step"] for p in first.logged] == [1, 2] and first.finished
    run1 = next((tmp_path / "runs").iterdir())
    trcli.run(cfg, resume=run1 / "step_00000002", max_steps=4, log=lambda *_: None)
    second = fake.runs[1]
    assert first.kw["resume"] == "allow" and second.kw["resume"] == "never"
    assert second.id != first.id
    steps = [p["trainer/step"] for p in second.logged]
    assert steps == [1, 2, 3, 4]                       # replayed prefix, then new steps
    assert second.summary.get("wandb/forked_from_step") == 2


def test_cli_resume_zero2_full_checkpointing_offload_is_exact(tmp_path):
    """4 steps in one go == 2 steps, then resume for 2 more (same losses)."""
    from nano_megatron_b200.cli import train as trcli
    from nano_megatron_b200.training.metric_history import read_metric_history

    over = dict(data_parallel={"mode": "zero2"},
                activation_checkpoint={"mode": "full", "offload_saved_tensors": True},
                offload={"optimizer_state": True})
    cfg_a = tmp_path / "a.yaml"
    cfg_a.write_text(yaml.safe_dump(_base_cfg(tmp_path / "a", **over)))
    trcli.run(cfg_a, max_steps=4, log=lambda *_: None)
    run_a = next((tmp_path / "a" / "runs").iterdir())
    full = [r.metrics["loss"] for r in read_metric_history(run_a / "metrics.jsonl")]
    cfg_b = tmp_path / "b.yaml"
    cfg_b.write_text(yaml.safe_dump(_base_cfg(tmp_path / "b", **over)))
    trcli.run(cfg_b, max_steps=2, log=lambda *_: None)
    run_b1 = next((tmp_path / "b" / "runs").iterdir())
    trcli.run(cfg_b, resume=run_b1 / "step_00000002", max_steps=4, log=lambda *_: None)
    run_b2 = sorted((tmp_path / "b" / "runs").iterdir())[-1]
    resumed = [r.metrics["loss"] for r in read_metric_history(run_b2 / "metrics.jsonl")]
    assert len(full) == len(resumed) == 4
    for a, b in zip(full, resumed):
        assert abs(a - b) < 1e-6 * abs(a), (full, resumed)


def test_async_save_lets_training_continue_before_flush(tmp_path):
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = _base_cfg(tmp_path, checkpoint={"async_save": True})
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    ids = torch.randint(0, 128, (4, 17))
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    tr.train_step(batch)
    saved = {k: v.clone() for k, v in comps.model.state_dict().items()}
    path = tr.save_checkpoint()
    tr.train_step(batch)                                # training continues meanwhile
    tr.flush()
    assert (path / ".complete").is_file()
    state = torch.load(path / "model.pt")
    for k, v in saved.items():
        torch.testing.assert_close(state[k], v, rtol=0, atol=0)   # snapshot, not later values


def _expand_save(rank, world, root):
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = _base_cfg(Path(root), parallel={"data": world})
    d["checkpoint"]["directory"] = str(Path(root) / "ck")
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    if world == 1:
        ids = torch.randint(0, 128, (4, 17))
        tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        tr.save_checkpoint()
        return
    latest = ck.latest()
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        tr.load_checkpoint(latest)
    new_replica = comps.parallel.coordinate.dp == 1
    assert any("new data-parallel replica" in str(w.message) for w in caught) == new_replica


@pytest.mark.distributed
def test_dp_expansion_keeps_new_replica_rng_with_warning(tmp_path):
    run_ranks(1, _expand_save, str(tmp_path))
    run_ranks(2, _expand_save, str(tmp_path))


def _repro_rank(rank, world, layout):
    """Train the same 3 steps twice from scratch on this rank; everything must be bitwise equal."""
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    runs = []
    for _trial in range(2):
        d = _base_cfg(Path("."), **layout)
        d["model"]["dropout"] = 0.1                     # exercises the keyed dropout streams
        d["checkpoint"]["save_interval"] = 0
        cfg = config_from_dict(d)
        comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
        tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                     data_parallel=comps.data_parallel, rng=comps.rng)
        gen = torch.Generator().manual_seed(11)
        rows = 4 * 2 // comps.parallel.dp.size
        losses = []
        for _ in range(3):
            ids = torch.randint(0, 128, (rows, 17), generator=gen)
            out = tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
            losses.append((float(out["loss_sum"]), float(out["token_count"])))
        with comps.data_parallel.full_parameters():
            params = {k: v.detach().clone() for k, v in comps.model.state_dict().items()}
        runs.append((losses, params))
    (la, pa), (lb, pb) = runs
    assert la == lb, (la, lb)
    assert pa.keys() == pb.keys()
    for k in pa:
        assert torch.equal(pa[k], pb[k]), k


@pytest.mark.distributed
@pytest.mark.parametrize("layout", [
    {"parallel": {"tensor": 2, "sequence_parallel": True}},
    {"parallel": {"data": 2}, "data_parallel": {"mode": "zero2", "overlap_grad_reduce": True}},
], ids=["tp2_sp", "dp2_zero2_overlap"])
def test_training_is_bitwise_reproducible_gloo(layout):
    run_ranks(2, _repro_rank, layout)


def _phase_rank(rank, world):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = _base_cfg(Path("."), parallel={"data": world})
    d["training"]["log_interval"] = 2
    d["checkpoint"]["save_interval"] = 0
    d["checkpoint"]["save_final"] = False
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)

    def batches():
        g = torch.Generator().manual_seed(rank)
        while True:
            ids = torch.randint(0, 128, (4, 17), generator=g)
            yield {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}

    tr.bind_data_iterator(batches())
    lines = []
    tr.fit(max_steps=4, log=lines.append)
    m = tr.last_metrics
    phases = [m[f"time_{p}_ms"] for p in ("forward_backward", "grad_sync", "clip", "optimizer")]
    assert all(v > 0 for v in phases), m
    # Each phase is a max over ranks, so their sum bounds the slowest rank's step from above.
    assert m["time_step_ms"] <= sum(phases) * (1 + 1e-9) + 1e-6, m
    assert m["time_forward_backward_ms"] > m["time_clip_ms"]
    assert m["tokens_per_second_device"] > 0
    if rank == 0:
        assert len(lines) == 2 and "time_optimizer_ms=" in lines[-1]


@pytest.mark.distributed
def test_fit_logs_per_phase_device_times_gloo():
    run_ranks(2, _phase_rank)


def _router_rank(rank, world):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training.batch_router import BatchRouter
    from nano_megatron_b200.training.engine import build_training_components

    d = _base_cfg(Path("."), parallel={"tensor": world})
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    router = BatchRouter(comps.parallel)
    ids = torch.arange(4 * 17).view(4, 17)
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    for _ in range(2):
        out = router.route(batch if router.is_source else None)
        assert torch.equal(out["input_ids"], ids[:, :-1]) and torch.equal(out["labels"], ids[:, 1:])
    if router.is_source:   # a new layout fails on the source before anything is sent
        with pytest.raises(ValueError, match="layout changed"):
            router.route({"input_ids": ids[:2, :-1], "labels": ids[:2, 1:]})


@pytest.mark.distributed
def test_batch_router_sends_header_once_and_rejects_layout_change_gloo():
    run_ranks(2, _router_rank)


def _overlap_rank(rank, world):
    """Record the strategy's bucket all-reduces around one training step."""
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.data_parallel import strategies
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = _base_cfg(Path("."), parallel={"data": world},
                  data_parallel={"mode": "ddp", "overlap_grad_reduce": True,
                                 "bucket_bytes": 1 << 12})
    d["model"]["layers"] = 4
    d["training"]["gradient_accumulation_steps"] = 3
    cfg = config_from_dict(d)
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    dp = comps.data_parallel
    buckets = {b.grad_data.data_ptr(): b for b in dp.buffers.buckets}
    events = []
    state = {"finalizing": False}
    real = strategies.dist

    class _Work:
        def __init__(self, inner, idx):
            self.inner, self.idx, self.waits = inner, idx, 0

        def wait(self):
            self.waits += 1
            events.append(("wait", self.idx, state["finalizing"]))
            return self.inner.wait()

    class _Dist:
        def __getattr__(self, name):
            return getattr(real, name)

        def all_reduce(self, t, *a, async_op=False, **kw):
            b = buckets.get(t.data_ptr())
            out = real.all_reduce(t, *a, async_op=async_op, **kw)
            if b is None:
                return out
            events.append(("async" if async_op else "sync", b.index, state["finalizing"]))
            if async_op:
                w = _Work(out, b.index)
                works.append(w)
                return w
            return out

    works = []
    strategies.dist = _Dist()
    finalize = dp.finalize_gradients

    def tracked():
        state["finalizing"] = True
        try:
            finalize()
        finally:
            state["finalizing"] = False

    dp.finalize_gradients = tracked
    try:
        ids = torch.randint(0, 128, (6, 17), generator=torch.Generator().manual_seed(rank))
        tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    finally:
        strategies.dist = real
    from nano_megatron_b200.data_parallel.zero3 import unit_of_name

    names = {id(p): n for n, p in dp._named}
    outer = {b.index for b in dp.buffers.buckets if b.defer_until_finalize or
             unit_of_name(names[id(b.slices[0].parameter)]) == "outer"}
    layer_buckets = {b.index for b in dp.buffers.buckets} - outer
    launched = [i for kind, i, fin in events if kind == "async"]
    # every layer bucket starts exactly once, inside the last microbatch's backward
    assert sorted(launched) == sorted(layer_buckets) and layer_buckets, \
        (events, layer_buckets, outer)
    assert all(not fin for kind, _, fin in events if kind == "async")
    # layer by layer in the backward's order (last layer first)
    unit = {b.index: unit_of_name(names[id(b.slices[0].parameter)]) for b in dp.buffers.buckets}
    layers = [unit[i][2] for i in launched]
    assert layers == sorted(layers, reverse=True) and layers[0] > layers[-1]
    # finalize waits on each in-flight reduction exactly once, then reduces the outer
    # (embedding / final norm / head, and any tied) buckets synchronously
    assert all(w.waits == 1 for w in works)
    assert all(fin for kind, _, fin in events if kind == "wait")
    assert {i for kind, i, fin in events if kind == "sync"} == outer and outer
    assert all(fin for kind, _, fin in events if kind == "sync")


@pytest.mark.distributed
def test_overlap_reducer_starts_buckets_during_backward_and_waits_once_gloo():
    run_ranks(2, _overlap_rank)


def _bf16_reduce_rank(rank, world, mode):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    out = {}
    for reduce in ("float32", "bfloat16"):
        d = _base_cfg(Path("."), parallel={"data": world}, data_parallel={"mode": mode},
                      precision={"grad_reduce": reduce})
        cfg = config_from_dict(d)
        comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
        tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                     data_parallel=comps.data_parallel, rng=comps.rng)
        dp = comps.data_parallel
        ids = torch.randint(0, 128, (4, 17), generator=torch.Generator().manual_seed(rank))
        micro = tr._prepare_batch({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        dp.zero_grad()
        tr.schedule.forward_backward(micro)
        dp.finalize_gradients()
        reduced = torch.cat([sh["grad"] for sh in dp.shards]) if hasattr(dp, "shards") \
            else dp.buffers.grad_flat
        out[reduce] = reduced.clone()
    lo, hi = out["bfloat16"], out["float32"]
    # summed in bf16: every reduced value is a bf16 number; the fp32 sum generally is not
    assert torch.equal(lo, lo.to(torch.bfloat16).float())
    assert not torch.equal(hi, hi.to(torch.bfloat16).float())
    assert ((lo - hi).norm() / hi.norm()).item() < 1e-2


@pytest.mark.distributed
@pytest.mark.parametrize("mode", ["ddp", "zero2"])
def test_grad_reduce_dtype_is_the_wire_precision_gloo(mode):
    run_ranks(2, _bf16_reduce_rank, mode)
