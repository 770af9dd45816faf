"""Owner of the default process group (torch.distributed over NCCL or gloo).

Behaviour of the reference runtime (src/nano_megatron/distributed/runtime.py:
27-346): RANK / WORLD_SIZE / LOCAL_RANK come from the environment; device
``auto`` means CUDA when available; backend ``auto`` means NCCL on CUDA and
gloo on CPU; ``torch.cuda.set_device(local_rank)`` binds the GPU and no eager
``device_id`` is passed to ``init_process_group``; a single process without a
rendezvous skips c10d; an existing default group is adopted (and not destroyed).
"""

from __future__ import annotations

import os
from datetime import timedelta
from typing import Any


class DistributedRuntimeError(RuntimeError):
    pass


class DistributedUnavailableError(DistributedRuntimeError):
    pass


def _env_int(name: str, default: int, minimum: int = 0) -> int:
    raw = os.environ.get(name)
    if raw is None:
        return default
    try:
        value = int(raw)
    except ValueError as error:
        raise DistributedRuntimeError(f"{name} must be an integer, got {raw!r}") from error
    if value < minimum:
        raise DistributedRuntimeError(f"{name} must be >= {minimum}, got {value}")
    return value


class DistributedRuntime:
    def __init__(self, config) -> None:
        self.config = config
        self._active = False
        self._owns_pg = False
        self._rank = self._world = self._local = None
        self._backend: str | None = None
        self._device = None
        self._c10d = False

    # ------------------------------------------------------------------ lifecycle
    def initialize(self) -> "DistributedRuntime":
        if self._active:
            return self
        import torch
        import torch.distributed as dist

        rank = _env_int("RANK", 0)
        world = _env_int("WORLD_SIZE", 1, minimum=1)
        local = _env_int("LOCAL_RANK", rank)
        dev_type = self.config.device
        if dev_type == "auto":
            dev_type = "cuda" if torch.cuda.is_available() else "cpu"
        backend = self.config.backend
        if backend == "auto":
            backend = "nccl" if dev_type == "cuda" else "gloo"
        if dev_type == "cuda":
            if not torch.cuda.is_available():
                raise DistributedRuntimeError("distributed.device=cuda but CUDA is unavailable")
            n = torch.cuda.device_count()
            if not 0 <= local < n:
                raise DistributedRuntimeError(
                    f"LOCAL_RANK={local} is outside the {n} visible CUDA devices")
            torch.cuda.set_device(local)
            device = torch.device("cuda", local)
        else:
            device = torch.device(dev_type)
        if dist.is_available() and dist.is_initialized():
            r, w, b = dist.get_rank(), dist.get_world_size(), str(dist.get_backend())
            if "WORLD_SIZE" in os.environ and w != world:
                raise DistributedRuntimeError(f"existing process group world size {w} != "
                                              f"WORLD_SIZE {world}")
            if "RANK" in os.environ and r != rank:
                raise DistributedRuntimeError(f"existing process group rank {r} != RANK {rank}")
            if self.config.backend != "auto" and b != backend:
                raise DistributedRuntimeError(f"existing process group backend {b!r} != "
                                              f"requested {backend!r}")
            rank, world, backend = r, w, b
            self._c10d = True
        elif world > 1 or "MASTER_ADDR" in os.environ or self.config.init_method != "env://":
            try:
                dist.init_process_group(backend=backend, init_method=self.config.init_method,
                                        timeout=timedelta(minutes=self.config.timeout_minutes),
                                        rank=rank, world_size=world)
            except Exception as error:  # noqa: BLE001
                raise DistributedRuntimeError(
                    f"failed to initialize torch.distributed with backend={backend!r}, "
                    f"rank={rank}, world_size={world}: {error}") from error
            self._owns_pg = True
            self._c10d = True
        self._rank, self._world, self._local = rank, world, local
        self._backend, self._device = backend, device
        self._active = True
        return self

    def close(self) -> None:
        if not self._active:
            return
        if self._owns_pg:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()
        self._active = False
        self._owns_pg = False

    def __enter__(self) -> "DistributedRuntime":
        return self.initialize()

    def __exit__(self, *exc) -> None:
        self.close()

    # ------------------------------------------------------------------ properties
    def _need(self):
        if not self._active:
            raise DistributedRuntimeError("DistributedRuntime is not initialized")

    @property
    def rank(self) -> int:
        self._need()
        return self._rank

    @property
    def world_size(self) -> int:
        self._need()
        return self._world

    @property
    def local_rank(self) -> int:
        self._need()
        return self._local

    @property
    def backend(self) -> str:
        self._need()
        return self._backend

    @property
    def device(self):
        self._need()
        return self._device

    @property
    def is_primary(self) -> bool:
        return self.rank == 0

    @property
    def uses_process_group(self) -> bool:
        return self._c10d

    # ------------------------------------------------------------------ collectives
    def barrier(self, group: Any | None = None) -> None:
        if not self._c10d:
            return
        import torch.distributed as dist

        if self._backend == "nccl":
            dist.barrier(group=group, device_ids=[self._device.index])
        else:
            dist.barrier(group=group)

    def all_gather_object(self, obj: Any, group: Any | None = None) -> list[Any]:
        if not self._c10d:
            return [obj]
        import torch.distributed as dist

        size = dist.get_world_size(group)
        out: list[Any] = [None] * size
        dist.all_gather_object(out, obj, group=group)
        return out

    def new_group(self, ranks: tuple[int, ...], *, backend: str | None = None) -> Any | None:
        if len(ranks) <= 1 or not self._c10d:
            return None
        import torch.distributed as dist

        return dist.new_group(ranks=list(ranks), backend=backend or self._backend,
                              timeout=timedelta(minutes=self.config.timeout_minutes))

    def destroy_group(self, process_group: Any | None) -> None:
        if process_group is None or not self._c10d:
            return
        import torch.distributed as dist

        if dist.is_initialized():
            try:
                dist.destroy_process_group(process_group)
            except Exception:  # noqa: BLE001 - best effort on shutdown
                pass

    def create_device_mesh(self, ranks: tuple[int, ...], process_group: Any | None) -> Any:
        from torch.distributed.device_mesh import DeviceMesh

        dev = "cuda" if self._device.type == "cuda" else "cpu"
        if process_group is None:
            return DeviceMesh(dev, list(ranks))
        return DeviceMesh.from_group(process_group, dev)
