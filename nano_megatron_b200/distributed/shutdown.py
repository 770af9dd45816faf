"""Ordered teardown of a training job's device, peer-memory and communicator resources.

A process that trained with tensor parallelism holds three kinds of state that
outlive the last step and depend on one another:

* CUDA graphs of microbatches. A graph that captured NCCL collectives keeps the
  communicator's pending work referenced; ``destroy_process_group`` then waits for
  that work forever, so every such graph is released first.
* The symmetric (IPC-mapped) workspace of the fused TP collectives. Each rank maps
  every peer's buffer. A rank may only unmap a peer's buffer once that peer's
  kernels no longer store into it, and may only free its own buffer once no peer
  maps it any more: two barriers over the TP group fence those two points.
* Process groups: the parallel context's subgroups, then the default group.

:func:`shutdown` runs the steps in that order on every rank. Each step is skipped
when its object is absent (a 1-GPU job has no workspace and no subgroups), and
every step is attempted even if an earlier one raised; the first error is raised
at the end. The reference closes its group registry and then the runtime
(src/nano_megatron/parallel/registry.py:173-182,
src/nano_megatron/distributed/runtime.py:148-152); it has no graphs or peer
mappings to release.
"""

from __future__ import annotations

import gc
from typing import Any, Callable

STEPS = ("synchronize", "release_graphs", "tp_barrier_before_unmap", "unmap_peers",
         "tp_barrier_before_free", "free_own_buffer", "close_subgroups", "close_runtime")


def _tp_barrier(parallel, device) -> None:
    import torch.distributed as dist

    if parallel is None:
        return
    tp = parallel.tp
    if tp.size <= 1 or tp.process_group is None or not dist.is_initialized():
        return
    if device is not None and getattr(device, "type", None) == "cuda":
        dist.barrier(group=tp.process_group, device_ids=[device.index])
    else:
        dist.barrier(group=tp.process_group)


def _synchronize(device) -> None:
    import torch

    if device is not None and getattr(device, "type", None) == "cuda" and \
            torch.cuda.is_available():
        torch.cuda.synchronize(device)


def _release_graphs(trainer) -> None:
    release = getattr(trainer, "release_graphs", None)
    if callable(release):
        release()
    gc.collect()


def _detach_workspace(model, workspace) -> None:
    if model is None or workspace is None:
        return
    for m in model.modules():
        if getattr(m, "tp_workspace", None) is workspace:
            m.tp_workspace = None


def _group_barrier(group, device) -> None:
    import torch.distributed as dist

    if group is None or getattr(group, "size", 1) <= 1 or not dist.is_initialized():
        return
    pg = getattr(group, "process_group", None)
    if device is not None and getattr(device, "type", None) == "cuda":
        dist.barrier(group=pg, device_ids=[device.index])
    else:
        dist.barrier(group=pg)


def shutdown(*, trainer=None, model=None, workspace=None, parallel=None, runtime=None,
             device=None, heaps=(), record: Callable[[str], Any] | None = None) -> None:
    """Release everything in the documented order; see the module docstring.

    ``heaps``: further peer-mapped allocations as (heap, group) pairs (e.g. the
    data-parallel replica buffers); each is unmapped after a barrier over its group and
    freed after a second one, like the TP workspace.
    ``record`` (optional) is called with each step name as it runs, for tests.
    """
    if model is None and trainer is not None:
        model = getattr(trainer, "model", None)
    if device is None and runtime is not None:
        device = getattr(runtime, "device", None) if getattr(runtime, "_active", True) else None
    errors: list[BaseException] = []

    def step(name: str, fn: Callable[[], Any]) -> None:
        if record is not None:
            record(name)
        try:
            fn()
        except BaseException as error:  # noqa: BLE001 - keep tearing down, raise the first
            errors.append(error)

    step("synchronize", lambda: _synchronize(device))
    step("release_graphs", lambda: _release_graphs(trainer))
    step("synchronize", lambda: _synchronize(device))
    if workspace is not None:
        step("tp_barrier_before_unmap", lambda: _tp_barrier(parallel, device))
        step("unmap_peers", workspace.close)
        step("synchronize", lambda: _synchronize(device))
        step("tp_barrier_before_free", lambda: _tp_barrier(parallel, device))
        step("free_own_buffer", lambda: (_detach_workspace(model, workspace),
                                         workspace.release()))
    for heap, group in heaps:
        if heap is None:
            continue
        step("tp_barrier_before_unmap", lambda g=group: _group_barrier(g, device))
        step("unmap_peers", heap.close)
        step("synchronize", lambda: _synchronize(device))
        step("tp_barrier_before_free", lambda g=group: _group_barrier(g, device))
        step("free_own_buffer", heap.release)
    if parallel is not None:
        step("close_subgroups", parallel.close)
    if runtime is not None:
        step("close_runtime", runtime.close)
    if errors:
        raise errors[0]
