"""Host-side failure detection (CPU / gloo; no GPU fault is ever provoked).

* PeerHealth: a failure marker or a stale heartbeat of another rank raises PeerFailure
  before the next step;
* a gloo rank that dies mid-run: the survivor stops with an error (PeerFailure between
  steps, or the collective's own error) instead of waiting forever;
* a step that raises leaves the data loader at the last completed step;
* corrupt / incomplete checkpoints and an occupied incomplete target directory are
  rejected on every rank.
Reference counterparts: tests/distributed_cpu/test_checkpoint_rank_local.py:445-599
(injected write failure, preflight), src/nano_megatron/training/trainer.py:599-605
(loader rollback).
"""

from __future__ import annotations

import json
import os
import time

import pytest
import torch
import torch.distributed as dist

from dist_utils import run_ranks


def test_peer_health_failure_marker_and_stale_heartbeat(tmp_path):
    from nano_megatron_b200.distributed.health import PeerFailure, PeerHealth

    store = dist.FileStore(str(tmp_path / "store"), 3)
    h = [PeerHealth(store, r, 3, interval_s=0.05, stale_s=1.0) for r in range(3)]
    for x in h:
        x.beat()
    h[0].check()                                   # everyone healthy
    h[2].report_failure(RuntimeError("disk full"))
    with pytest.raises(PeerFailure, match="rank 2: disk full"):
        h[0].check()
    h[1].beat()
    with pytest.raises(PeerFailure, match="rank 1 silent"):
        h[2].check(now=time.time() + 10.0)
    h[0].start()
    time.sleep(0.2)
    h[0].stop()


def _dying_worker(rank, world, out_dir):
    from nano_megatron_b200.distributed.health import PeerFailure, PeerHealth
    from torch.distributed import distributed_c10d as c10d

    health = PeerHealth(c10d._get_default_store(), rank, world, interval_s=0.05,
                        stale_s=30.0).start()
    x = torch.ones(4)
    for step in range(50):
        if rank == 1 and step == 3:
            health.report_failure(RuntimeError("injected failure on rank 1"))
            os._exit(0)                              # leaves between steps, nothing in flight
        try:
            health.check()
            dist.all_reduce(x)
        except (PeerFailure, RuntimeError) as e:     # noqa: PERF203
            with open(os.path.join(out_dir, "survivor.json"), "w") as f:
                json.dump({"rank": rank, "step": step, "error": str(e)[:300],
                           "peer_failure": isinstance(e, PeerFailure)}, f)
            os._exit(0)
        time.sleep(0.1)


def test_survivor_stops_when_a_rank_dies(tmp_path):
    from dist_utils import _entry

    ctx = torch.multiprocessing.get_context("spawn")
    errq = ctx.SimpleQueue()
    init = tmp_path / "rdzv"
    procs = [ctx.Process(target=_entry, args=(r, 2, str(init), _dying_worker, (str(tmp_path),),
                                               errq)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert time.time() - t0 < 120
    rep = json.loads((tmp_path / "survivor.json").read_text())
    assert rep["rank"] == 0 and rep["step"] >= 3
    assert "rank 1" in rep["error"] or not rep["peer_failure"]


def test_failed_step_rolls_back_the_data_position(tmp_path):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.data import StatefulDataLoader
    from nano_megatron_b200.data.datasets import RandomTokenDataset
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    cfg = config_from_dict({
        "model": {"layers": 1, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 4,
                  "seq_length": 16, "vocab_size": 64},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "precision": {"params": "float32", "compute": "float32"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 1, "max_steps": 5}})
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    ds = RandomTokenDataset(num_samples=64, sequence_length=16, vocab_size=64, seed=1)
    loader = StatefulDataLoader(ds, local_batch_size=2, replica_count=1, replica_index=0,
                                shuffle=True, shuffle_seed=1, data_fingerprint=ds.fingerprint)
    tr.bind_data_iterator(loader, data_fingerprint=ds.fingerprint)
    real = tr.train_step
    calls = {"n": 0}

    def flaky(batch):
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("injected step failure")
        return real(batch)

    tr.train_step = flaky
    with pytest.raises(RuntimeError, match="injected"):
        tr.fit(max_steps=5, log=None)
    assert tr.state.step == 2
    assert loader.state_dict()["sample_offset"] == 4      # two completed steps x 2 samples


def test_corrupt_and_incomplete_checkpoints_are_rejected(tmp_path):
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    cfg = config_from_dict({
        "model": {"layers": 1, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 4,
                  "seq_length": 16, "vocab_size": 64},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "precision": {"params": "float32", "compute": "float32"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 1},
        "checkpoint": {"directory": str(tmp_path / "ck")}})
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    ids = torch.randint(0, 64, (2, 17))
    tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    path = tr.save_checkpoint()
    (path / "manifest.json").write_text("{ not json")
    with pytest.raises(ValueError):
        tr.load_checkpoint(path)
    (path / ".complete").unlink()
    with pytest.raises(FileNotFoundError, match="incomplete"):
        tr.load_checkpoint(path)
    busy = tmp_path / "ck" / "step_00000009"
    busy.mkdir(parents=True)
    (busy / "leftover.pt").write_bytes(b"x")
    with pytest.raises(RuntimeError, match="incomplete checkpoint directory already exists"):
        ck.save(9, model=comps.model, data_parallel=comps.data_parallel,
                trainer_state=tr.state.state_dict())


def _preflight_worker(rank, world, root):
    from pathlib import Path

    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    cfg = config_from_dict({
        "model": {"layers": 1, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 4,
                  "seq_length": 16, "vocab_size": 64},
        "parallel": {"data": 2},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "precision": {"params": "float32", "compute": "float32"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 1},
        "checkpoint": {"directory": root}})
    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    if rank == 0:
        busy = Path(root) / "step_00000000"
        busy.mkdir(parents=True, exist_ok=True)
        (busy / "leftover.pt").write_bytes(b"x")
    dist.barrier()
    with pytest.raises(RuntimeError, match="preflight failed"):
        tr.save_checkpoint()                # rank 1 learns of rank 0's refusal


@pytest.mark.distributed
def test_preflight_error_reaches_every_rank(tmp_path):
    run_ranks(2, _preflight_worker, str(tmp_path / "ck"))
