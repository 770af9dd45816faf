"""Materialise a :class:`GroupPlan` into communicators.

Every rank must call ``new_group`` for every planned group in one global
order (a c10d requirement), including groups it is not a member of. Identical
(ranks, backend, channel) triples share one communicator; size-one groups reuse
the default channel and never create a communicator. Reference:
src/nano_megatron/parallel/registry.py:38-191.
"""

from __future__ import annotations

from typing import Any, Protocol

from .group import ParallelGroup
from .group_plan import GroupKeyLike, GroupPlan, normalize_group_key
from .topology import ParallelTopology


class GroupRuntime(Protocol):
    rank: int
    world_size: int
    backend: str

    def new_group(self, ranks: tuple[int, ...], *, backend: str | None = None) -> Any | None: ...

    def destroy_group(self, process_group: Any | None) -> None: ...


class ParallelGroupRegistry:
    def __init__(self, runtime: GroupRuntime, topology: ParallelTopology) -> None:
        if runtime.world_size != topology.world_size:
            raise ValueError(f"runtime world size {runtime.world_size} does not match topology "
                             f"world size {topology.world_size}")
        self._runtime = runtime
        self._topology = topology
        self._plan: GroupPlan | None = None
        self._groups: dict[GroupKeyLike, ParallelGroup] = {}
        self._families: dict[GroupKeyLike, tuple[tuple[int, ...], ...]] = {}
        self._resources: dict[tuple, Any] = {}
        self._meshes: dict[GroupKeyLike, Any] = {}
        self._closed = False

    plan = property(lambda self: self._plan)
    topology = property(lambda self: self._topology)
    resource_count = property(lambda self: len(self._resources))

    def materialize(self, plan: GroupPlan) -> "ParallelGroupRegistry":
        self._require_open()
        if self._plan is not None:
            raise RuntimeError("group registry was already materialized")
        me = self._runtime.rank
        for spec in plan:
            family = []
            for planned in GroupPlan.expand_spec(self._topology, spec):
                ranks = tuple(sorted(planned.ranks))
                family.append(ranks)
                backend = spec.backend or self._runtime.backend
                channel = spec.channel if len(ranks) > 1 else "default"
                key = (ranks, backend, channel)
                if len(ranks) > 1 and key not in self._resources:
                    self._resources[key] = self._runtime.new_group(ranks, backend=spec.backend)
                if me in ranks:
                    self._groups[spec.key] = ParallelGroup(
                        key=spec.key, ranks=ranks,
                        process_group=self._resources.get(key) if len(ranks) > 1 else None,
                        rank=ranks.index(me), size=len(ranks), backend=backend, channel=channel)
            self._families[spec.key] = tuple(family)
        self._plan = plan
        return self

    def has_group(self, key: GroupKeyLike) -> bool:
        return normalize_group_key(key) in self._groups

    def group(self, key: GroupKeyLike) -> ParallelGroup:
        self._require_open()
        k = normalize_group_key(key)
        if k not in self._groups:
            raise KeyError(f"rank {self._runtime.rank} is not a member of a {k!s} group")
        return self._groups[k]

    def family(self, key: GroupKeyLike) -> tuple[tuple[int, ...], ...]:
        return self._families[normalize_group_key(key)]

    def group_ranks_for_rank(self, key: GroupKeyLike, rank: int) -> tuple[int, ...] | None:
        for ranks in self.family(key):
            if rank in ranks:
                return ranks
        return None

    def mesh(self, key: GroupKeyLike) -> Any:
        k = normalize_group_key(key)
        if k not in self._meshes:
            group = self.group(k)
            factory = getattr(self._runtime, "create_device_mesh", None)
            if factory is None:
                raise RuntimeError("runtime cannot create device meshes")
            self._meshes[k] = factory(group.ranks, group.process_group)
        return self._meshes[k]

    def close(self) -> None:
        if self._closed:
            return
        for pg in self._resources.values():
            if pg is not None:
                self._runtime.destroy_group(pg)
        self._resources.clear()
        self._groups.clear()
        self._meshes.clear()
        self._closed = True

    def _require_open(self) -> None:
        if self._closed:
            raise RuntimeError("group registry is closed")


GroupRegistry = ParallelGroupRegistry
