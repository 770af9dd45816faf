"""Ordered teardown of a tensor-parallel job (distributed/shutdown.py).

The order is what keeps a multi-GPU process from hanging at exit: CUDA graphs that
captured NCCL work go before any process group; peers unmap each other's symmetric
buffers only after a TP barrier, and free their own buffer only after a second one;
subgroups go before the default group. A recording stand-in checks the order on one
process; two gloo ranks run the real path through ``TrainingComponents.close``.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from nano_megatron_b200.distributed.shutdown import shutdown
from tests.dist_utils import run_ranks


class _Recorder:
    def __init__(self):
        self.events: list[str] = []


class _Workspace:
    def __init__(self, rec):
        self.rec = rec

    def close(self):
        self.rec.events.append("ws.close")

    def release(self):
        self.rec.events.append("ws.release")


class _Trainer:
    def __init__(self, rec):
        self.rec = rec
        self.model = torch.nn.Linear(2, 2)

    def release_graphs(self):
        self.rec.events.append("trainer.release_graphs")


class _Parallel:
    def __init__(self, rec):
        self.rec = rec
        self.tp = SimpleNamespace(size=1, process_group=None)

    def close(self):
        self.rec.events.append("parallel.close")


class _Runtime:
    def __init__(self, rec):
        self.rec = rec
        self.device = torch.device("cpu")

    def close(self):
        self.rec.events.append("runtime.close")


def test_shutdown_order_with_workspace():
    rec = _Recorder()
    steps: list[str] = []
    shutdown(trainer=_Trainer(rec), workspace=_Workspace(rec), parallel=_Parallel(rec),
             runtime=_Runtime(rec), record=steps.append)
    assert rec.events == ["trainer.release_graphs", "ws.close", "ws.release", "parallel.close",
                          "runtime.close"]
    assert steps == ["synchronize", "release_graphs", "synchronize", "tp_barrier_before_unmap",
                     "unmap_peers", "synchronize", "tp_barrier_before_free",
                     "free_own_buffer", "close_subgroups", "close_runtime"]


def test_shutdown_without_workspace_skips_peer_steps():
    rec = _Recorder()
    steps: list[str] = []
    shutdown(trainer=_Trainer(rec), parallel=_Parallel(rec), runtime=_Runtime(rec),
             record=steps.append)
    assert rec.events == ["trainer.release_graphs", "parallel.close", "runtime.close"]
    assert "unmap_peers" not in steps and "free_own_buffer" not in steps


def test_shutdown_continues_after_a_failing_step_and_raises_the_first_error():
    rec = _Recorder()

    class Bad(_Workspace):
        def close(self):
            rec.events.append("ws.close")
            raise RuntimeError("unmap failed")

    with pytest.raises(RuntimeError, match="unmap failed"):
        shutdown(trainer=_Trainer(rec), workspace=Bad(rec), parallel=_Parallel(rec),
                 runtime=_Runtime(rec))
    # later steps still ran: the groups are destroyed even when a peer unmap failed
    assert rec.events[-2:] == ["parallel.close", "runtime.close"]


def test_graph_release_drops_captured_graphs():
    from nano_megatron_b200.pipeline_parallel.schedules.no_pipeline import NoPipelineSchedule

    released = []

    class G:
        def release(self):
            released.append(1)

    sched = NoPipelineSchedule(stage=None, data_parallel=None, use_graphs=True)
    sched._graphs = {"a": G(), "b": G()}
    sched.release_graphs()
    assert sched._graphs == {} and len(released) == 2


def _tp2_components_close(rank, world):
    import torch.distributed as dist

    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    cfg = config_from_dict({
        "distributed": {"backend": "gloo", "device": "cpu"},
        "parallel": {"tensor": 2, "sequence_parallel": True},
        "model": {"layers": 1, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 2,
                  "kv_heads": 2, "seq_length": 16, "vocab_size": 64},
        "precision": {"params": "float32", "compute": "float32", "grad_reduce": "float32"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 1}})
    runtime = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, runtime)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    ids = torch.randint(0, 64, (2, 17), generator=torch.Generator().manual_seed(0))
    tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    # a stand-in workspace: the real one needs CUDA IPC; the TP barriers around it are real
    events = []
    comps.tp_workspace = SimpleNamespace(close=lambda: events.append("close"),
                                         release=lambda: events.append("release"))
    comps.close(tr, keep_runtime=True)
    assert events == ["close", "release"]
    assert comps.tp_workspace is None
    with pytest.raises(RuntimeError):
        comps.parallel.tp          # the registry is closed: subgroups are gone
    assert dist.is_initialized()   # keep_runtime leaves the default group to the harness


@pytest.mark.distributed
def test_components_close_on_two_gloo_ranks():
    run_ranks(2, _tp2_components_close, timeout=240)
