"""DistributedRuntime environment semantics with a recording torch.distributed stand-in.

Counterpart of the reference's runtime unit tests (tests/unit/test_distributed_runtime.py:
13-141): rank / world / local rank from the environment, ``auto`` backend and device
resolution, no eager ``device_id`` passed to ``init_process_group``, no rendezvous for a
single process without one, adoption (not destruction) of an existing default group, and
clear errors for inconsistent environments.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from nano_megatron_b200.distributed import runtime as rt_mod


class _Recorder:
    def __init__(self, *, initialized=False, rank=0, world=1, backend="gloo"):
        self.calls = []
        self._init = initialized
        self._rank, self._world, self._backend = rank, world, backend

    def is_available(self):
        return True

    def is_initialized(self):
        return self._init

    def init_process_group(self, **kw):
        self.calls.append(("init", kw))
        self._init = True

    def destroy_process_group(self):
        self.calls.append(("destroy",))
        self._init = False

    def get_rank(self):
        return self._rank

    def get_world_size(self):
        return self._world

    def get_backend(self):
        return self._backend


def _cfg(**kw):
    base = dict(backend="auto", device="cpu", init_method="env://", timeout_minutes=3)
    base.update(kw)
    return SimpleNamespace(**base)


@pytest.fixture
def fake(monkeypatch):
    rec = _Recorder()
    monkeypatch.setattr(torch, "distributed", rec)
    import sys

    monkeypatch.setitem(sys.modules, "torch.distributed", rec)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        monkeypatch.delenv(k, raising=False)
    return rec


def test_single_process_without_rendezvous_skips_c10d(fake):
    r = rt_mod.DistributedRuntime(_cfg()).initialize()
    assert (r.rank, r.world_size, r.local_rank) == (0, 1, 0) and fake.calls == []
    r.close()
    assert fake.calls == []


def test_env_ranks_auto_backend_and_no_eager_device_id(fake, monkeypatch):
    monkeypatch.setenv("RANK", "3")
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("LOCAL_RANK", "1")
    r = rt_mod.DistributedRuntime(_cfg()).initialize()
    (name, kw), = fake.calls
    assert name == "init" and kw["backend"] == "gloo" and kw["rank"] == 3
    assert kw["world_size"] == 4 and "device_id" not in kw
    assert kw["timeout"].total_seconds() == 180 and kw["init_method"] == "env://"
    assert (r.rank, r.world_size, r.local_rank) == (3, 4, 1)
    r.close()
    assert fake.calls[-1] == ("destroy",)          # the runtime owned the group


def test_existing_group_is_adopted_and_not_destroyed(fake, monkeypatch):
    fake._init, fake._rank, fake._world, fake._backend = True, 1, 2, "gloo"
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    r = rt_mod.DistributedRuntime(_cfg()).initialize()
    assert (r.rank, r.world_size) == (1, 2) and fake.calls == []
    r.close()
    assert fake.calls == []


@pytest.mark.parametrize("env,message", [
    ({"WORLD_SIZE": "0"}, "WORLD_SIZE must be >= 1"),
    ({"RANK": "x"}, "RANK must be an integer"),
])
def test_bad_environment_is_rejected(fake, monkeypatch, env, message):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    with pytest.raises(rt_mod.DistributedRuntimeError, match=message):
        rt_mod.DistributedRuntime(_cfg()).initialize()


def test_existing_group_must_match_the_environment(fake, monkeypatch):
    fake._init, fake._rank, fake._world = True, 0, 2
    monkeypatch.setenv("WORLD_SIZE", "4")
    with pytest.raises(rt_mod.DistributedRuntimeError, match="world size"):
        rt_mod.DistributedRuntime(_cfg()).initialize()


def test_cuda_requested_without_cuda_is_an_error(fake, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(rt_mod.DistributedRuntimeError, match="CUDA is unavailable"):
        rt_mod.DistributedRuntime(_cfg(device="cuda")).initialize()
