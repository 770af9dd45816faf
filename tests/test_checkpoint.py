"""Checkpoint save/resume (CPU, gloo).

* single process: save after a step, scramble, load, and the next step's loss
  and parameters match an uninterrupted run exactly (reference:
  tests/integration/test_checkpoint_resume.py);
* 4 gloo ranks TP2xDP2 ZeRO-1 save -> 2 ranks TP2xDP1 load (data-parallel
  reshard), parameters and optimizer masters equal;
* a write failure on one rank is raised on every rank and no ``.complete`` is
  published; retention keeps ``keep_last`` plus the pinned best checkpoint.
"""

from __future__ import annotations

import os

import pytest
import torch

from dist_utils import run_ranks

MODEL = {"layers": 2, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 4, "kv_heads": 2,
         "seq_length": 16, "vocab_size": 128}


def _cfg(tmp, *, tp=1, dp=1, mode="ddp", keep_last=2, async_save=False):
    from nano_megatron_b200.config import config_from_dict

    return config_from_dict({
        "model": dict(MODEL),
        "parallel": {"tensor": tp, "pipeline": 1, "context": 1, "expert": 1, "data": dp,
                     "sequence_parallel": False},
        "precision": {"params": "float32", "compute": "float32"},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 4 // (2 * dp)},
        "data_parallel": {"mode": mode},
        "optimizer": {"lr": 1e-2, "clip_grad_norm": 1.0},
        "checkpoint": {"directory": str(tmp), "keep_last": keep_last,
                       "async_save": async_save}})


def _batch(step):
    g = torch.Generator().manual_seed(1000 + step)
    ids = torch.randint(0, MODEL["vocab_size"], (4, MODEL["seq_length"] + 1), generator=g)
    return {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous()}


def _build(cfg):
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    rt = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, rt)
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    return comps, tr


def _loss(out):
    return float(out["loss_sum"] / out["token_count"])


def _local(batch, parallel):
    rows = 4 // parallel.dp.size
    r = parallel.coordinate.dp
    return {k: v[r * rows:(r + 1) * rows] for k, v in batch.items()}


def test_single_process_exact_resume(tmp_path):
    torch.manual_seed(0)
    cfg = _cfg(tmp_path / "ck", async_save=True)
    comps, tr = _build(cfg)
    tr.train_step(_batch(0))
    path = tr.save_checkpoint()
    tr.flush()
    assert (path / ".complete").is_file() and (path / "model.pt").is_file()
    ref_loss = _loss(tr.train_step(_batch(1)))
    ref_params = {k: v.detach().clone() for k, v in comps.model.state_dict().items()}

    torch.manual_seed(123)
    comps2, tr2 = _build(_cfg(tmp_path / "ck"))
    assert tr2.checkpoint.latest() == path
    tr2.load_checkpoint(path)
    assert tr2.state.step == 1
    loss = _loss(tr2.train_step(_batch(1)))
    assert loss == pytest.approx(ref_loss, rel=0, abs=1e-6)
    for k, v in comps2.model.state_dict().items():
        torch.testing.assert_close(v, ref_params[k], rtol=0, atol=1e-6)
    # the reference's manifest schema and file layout
    import json

    man = json.loads((path / "manifest.json").read_text())
    assert man["schema_version"] == 2 and man["storage_backend"] == "torch.save"
    assert (path / "trainer_state.pt").is_file() and (path / "data_parallel.pt").is_file()


def test_retention_and_best_validation_pin(tmp_path):
    cfg = _cfg(tmp_path / "ck", keep_last=1)
    comps, tr = _build(cfg)
    paths = []
    for s in range(3):
        tr.train_step(_batch(s))
        paths.append(tr.save_checkpoint())
        if s == 0:
            tr.checkpoint.pin_best_validation(tr.state.step, 3.5)
    left = sorted(p.name for p in (tmp_path / "ck").glob("step_*"))
    assert left == [paths[0].name, paths[2].name]
    assert tr.checkpoint.best_validation()["checkpoint"] == paths[0].name


def _reshard_save(rank, world, root, mode="zero1"):
    cfg = _cfg(root, tp=2, dp=2, mode=mode)
    comps, tr = _build(cfg)
    for s in range(2):
        tr.train_step(_local(_batch(s), comps.parallel))
    tr.save_checkpoint()
    with comps.data_parallel.full_parameters():
        params = {k: v.clone() for k, v in comps.model.state_dict().items()}
    st = {"params": params, "dp": comps.data_parallel.state_dict()}
    if comps.parallel.coordinate.dp == 0:
        torch.save(st, os.path.join(root, f"expect_tp{comps.parallel.coordinate.tp}.pt"))


def _reshard_load(rank, world, root, mode="zero1"):
    cfg = _cfg(root, tp=2, dp=1, mode=mode)
    comps, tr = _build(cfg)
    tr.load_checkpoint(tr.checkpoint.latest())
    exp = torch.load(os.path.join(root, f"expect_tp{comps.parallel.coordinate.tp}.pt"))
    with comps.data_parallel.full_parameters():
        got = {k: v.clone() for k, v in comps.model.state_dict().items()}
    for k, v in got.items():
        torch.testing.assert_close(v, exp["params"][k], rtol=0, atol=0)
    got = comps.data_parallel.state_dict()
    for b, e in exp["dp"]["buckets"].items():
        for key in ("master_parameter", "exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(got["buckets"][b][key], e[key], rtol=0, atol=0)
    assert tr.state.step == 2
    tr.train_step(_local(_batch(2), comps.parallel))


@pytest.mark.distributed
@pytest.mark.parametrize("mode", ["zero1", "zero3"])
def test_zero_dp_reshard_gloo(tmp_path, mode):
    root = str(tmp_path)
    run_ranks(4, _reshard_save, root, mode)
    run_ranks(2, _reshard_load, root, mode)


def _failing_save(rank, world, root):
    from nano_megatron_b200.checkpoint import manager as mgr

    cfg = _cfg(root, dp=2)
    comps, tr = _build(cfg)
    tr.train_step(_local(_batch(0), comps.parallel))
    if rank == 1:
        def boom(payloads):
            raise OSError("disk full (injected)")
        mgr._write_payloads = boom
    with pytest.raises(RuntimeError, match="disk full"):
        tr.save_checkpoint()
    assert not (tmp_path_step(root) / ".complete").exists()


def tmp_path_step(root):
    from pathlib import Path

    return Path(root) / "step_00000001"


@pytest.mark.distributed
def test_write_failure_is_collective_gloo(tmp_path):
    run_ranks(2, _failing_save, str(tmp_path))


def test_fsdp2_layout_round_trip_of_zero_bucket_state():
    """Flat ZeRO bucket state -> the reference's per-parameter FSDP2 layout -> back."""
    from types import SimpleNamespace

    from nano_megatron_b200.checkpoint.fsdp2_format import from_fsdp2_state, to_fsdp2_state

    shapes = {"model.embedding.weight": (6, 4), "model.layers.0.input_norm.weight": (4,),
              "model.final_norm.weight": (4,)}
    names = list(shapes)
    sizes = [int(torch.tensor(shapes[n]).prod()) for n in names]

    def bucket(index, members):
        slices, cur = [], 0
        for n in members:
            k = sizes[names.index(n)]
            slices.append(SimpleNamespace(name=n, start=cur, end=cur + k))
            cur += k
        return SimpleNamespace(index=index, slices=slices, numel=cur,
                               metadata=lambda m=members, c=cur: {"parameter_names": list(m),
                                                                  "numel": c})

    buckets = [bucket(0, names[:2]), bucket(1, names[2:])]
    g = torch.Generator().manual_seed(0)
    model = {n: torch.randn(shapes[n], generator=g) for n in names}
    model["model.lm_head.weight"] = model["model.embedding.weight"]       # tied view
    dp = {"mode": "zero3", "step": 7, "learning_rate": 1e-3, "buckets": {}}
    for b in buckets:
        dp["buckets"][str(b.index)] = {
            "metadata": b.metadata(),
            "master_parameter": torch.cat([model[s.name].reshape(-1) for s in b.slices]),
            "exp_avg": torch.randn(b.numel, generator=g),
            "exp_avg_sq": torch.rand(b.numel, generator=g)}
    nested = to_fsdp2_state(model, dp, buckets, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    group = nested["optimizer"]["param_groups"][0]
    assert group["params"] == names and group["lr"] == 1e-3 and group["betas"] == (0.9, 0.95)
    assert set(nested["optimizer"]["state"]) == set(names)         # the tied head once
    assert float(nested["optimizer"]["state"][names[0]]["step"]) == 7.0
    back = from_fsdp2_state(nested, buckets)
    assert back["step"] == 7 and back["learning_rate"] == 1e-3
    for k, entry in dp["buckets"].items():
        for key in ("master_parameter", "exp_avg", "exp_avg_sq"):
            assert torch.equal(back["buckets"][k][key], entry[key]), (k, key)
