"""Pipeline executor ordering with a recording communicator (no process group).

Mirrors the reference's executor unit tests (tests/unit/test_pipeline_schedule_executor.py,
tests/unit/test_pipeline_p2p.py): for every schedule, stage and microbatch count the
executor posts exactly the receives and issues exactly the sends its plan implies, in plan
order, with a bounded number of sends in flight (with or without ``overlap_p2p``); the
gradient-synchronising forward and the last backward of each chunk are flagged to the
data-parallel strategy exactly once.
"""

from __future__ import annotations

from contextlib import contextmanager
from types import SimpleNamespace

import pytest
import torch

from nano_megatron_b200.pipeline_parallel.schedules.executor import PipelineScheduleExecutor

SHAPE = (3, 2, 4)


class _Work:
    def __init__(self, log, tag):
        self.log, self.tag = log, tag
        self.done = False

    def wait(self):
        self.done = True


class _Recorder:
    """Stands in for the P2P communicator and records every call."""

    def __init__(self):
        self.ops: list = []
        self.in_flight: list = []
        self.after_action: list = []

    def _send(self, kind, t, dst):
        self.ops.append((kind, dst))
        self.in_flight.append(_Work(self.ops, kind))

    def send_activation(self, t, dst, microbatch=0, chunk=0):
        self._send("send_act", t, dst)

    def send_grad(self, t, dst, microbatch=0, chunk=0):
        self._send("send_grad", t, dst)

    def post_recv_activation(self, shape, src, microbatch=0, chunk=0):
        self.ops.append(("recv_act", src))
        return _Work(self.ops, "recv"), torch.ones(shape)

    def post_recv_grad(self, shape, src, microbatch=0, chunk=0):
        self.ops.append(("recv_grad", src))
        return _Work(self.ops, "recv"), torch.ones(shape)

    def drain_sends(self, keep=0):
        while len(self.in_flight) > keep:
            self.in_flight.pop(0).wait()
        self.after_action.append(len(self.in_flight))

    def warmup(self):
        pass


class _Stage(torch.nn.Module):
    def __init__(self, last: bool):
        super().__init__()
        self.w = torch.nn.Parameter(torch.full(SHAPE[-1:], 0.5))
        self.last = last

    def forward(self, inp, mb):
        x = mb["x"] if inp is None else inp
        y = x * self.w
        return y.square().mean() if self.last else y


class _Model(torch.nn.Module):
    def __init__(self, stages):
        super().__init__()
        self.stages = torch.nn.ModuleList(stages)

    def chunk(self, c):
        return self.stages[c]


class _DP:
    def __init__(self):
        self.forward_sync: list = []
        self.last_backward: list = []

    @contextmanager
    def forward_microbatch_context(self, *, synchronize_gradients, unit=None):
        self.forward_sync.append(bool(synchronize_gradients))
        yield

    @contextmanager
    def microbatch_context(self, *, is_last_microbatch, unit=None):
        self.last_backward.append(bool(is_last_microbatch))
        yield


def _executor(schedule, pp, rank, chunks, overlap):
    parallel = SimpleNamespace(pp=SimpleNamespace(size=pp, ranks=list(range(pp))),
                               coordinate=SimpleNamespace(pp=rank), rank=rank,
                               group=lambda key: (_ for _ in ()).throw(KeyError(key)))
    stages = [_Stage(last=(c * pp + rank == pp * chunks - 1)) for c in range(chunks)]
    dp = _DP()
    ex = PipelineScheduleExecutor(model=_Model(stages), parallel=parallel, data_parallel=dp,
                                  schedule=schedule, chunks=chunks, activation_shape=SHAPE,
                                  dtype=torch.float32, device=torch.device("cpu"),
                                  overlap_p2p=overlap)
    ex.p2p = _Recorder()
    ex._warm = True
    return ex, dp


def _expected_ops(ex, plan):
    ops = []
    for a in plan:
        first, last = ex._is_first(a.chunk), ex._is_last(a.chunk)
        if a.kind == "F":
            if not first:
                ops.append(("recv_act", ex.rank - 1))
            if not last:
                ops.append(("send_act", ex.rank + 1))
        else:
            if not last:
                ops.append(("recv_grad", ex.rank + 1))
            if not first:
                ops.append(("send_grad", ex.rank - 1))
    return ops


CASES = [("gpipe", 2, r, 1, m) for r in range(2) for m in (1, 3)] + \
        [("1f1b", 4, r, 1, m) for r in range(4) for m in (2, 6)] + \
        [("interleaved_1f1b", 2, r, 2, m) for r in range(2) for m in (2, 4)]


@pytest.mark.parametrize("overlap", [True, False], ids=["overlap", "sync"])
@pytest.mark.parametrize("schedule,pp,rank,chunks,m", CASES)
def test_executor_issues_the_plans_transfers_in_order(schedule, pp, rank, chunks, m, overlap):
    ex, dp = _executor(schedule, pp, rank, chunks, overlap)
    mbs = [{"x": torch.randn(SHAPE), "labels": torch.zeros(SHAPE[:2], dtype=torch.long)}
           for _ in range(m)]
    plan = ex.plan(m, forward_only=False)
    acc = ex.forward_backward(mbs)
    rec = ex.p2p
    assert rec.ops == _expected_ops(ex, plan)
    assert rec.in_flight == []                      # everything drained at the end
    assert max(rec.after_action) <= 4                # a bounded number of sends in flight
    # data-parallel flags: one gradient-synchronising forward and one last backward per
    # chunk, and the synchronising forward belongs to the last backward's microbatch
    assert sum(dp.last_backward) == chunks and sum(dp.forward_sync) == chunks
    last_f = [a for a in plan if a.kind == "F"]
    last_b = {}
    for a in plan:
        if a.kind == "B":
            last_b[a.chunk] = a.microbatch
    flagged = [(a.chunk, a.microbatch) for a, s in zip(last_f, dp.forward_sync) if s]
    assert sorted(flagged) == sorted(last_b.items())
    if any(ex._is_last(c) for c in range(chunks)):
        assert acc.token_count is not None and float(acc.token_count) == m * SHAPE[0] * SHAPE[1]


def test_forward_only_sends_no_gradients():
    ex, dp = _executor("1f1b", 2, 0, 1, True)
    mbs = [{"x": torch.randn(SHAPE), "labels": torch.zeros(SHAPE[:2], dtype=torch.long)}
           for _ in range(3)]
    ex.forward_backward(mbs, forward_only=True)
    assert ex.p2p.ops == [("send_act", 1)] * 3
    assert dp.last_backward == [] and dp.forward_sync == []
