"""Immutable per-rank view of the parallel topology and its process groups.

Parallel state is injected explicitly (no module-level singleton), as in the
reference (src/nano_megatron/parallel/context.py:26-175).
"""

from __future__ import annotations

from typing import Any

from .axes import ParallelAxis, ParallelCoordinate
from .group import ParallelGroup
from .group_plan import DEFAULT_GROUP_PLAN, GroupKey, GroupKeyLike, GroupPlan
from .registry import ParallelGroupRegistry
from .topology import ParallelTopology

_AXIS_KEYS = {
    ParallelAxis.TP: GroupKey.TP,
    ParallelAxis.PP: GroupKey.PP,
    ParallelAxis.CP: GroupKey.CP,
    ParallelAxis.EP: GroupKey.EP,
    ParallelAxis.DP: GroupKey.DP_AXIS,
}


class ParallelContext:
    def __init__(self, *, topology: ParallelTopology, registry: ParallelGroupRegistry,
                 rank: int, sequence_parallel: bool = False) -> None:
        self.topology = topology
        self.registry = registry
        self._rank = rank
        self._sequence_parallel = bool(sequence_parallel)
        self.coordinate: ParallelCoordinate = topology.rank_to_coordinate(rank)

    @classmethod
    def create(cls, runtime, parallel_config, *, group_plan: GroupPlan | None = None
               ) -> "ParallelContext":
        topology = ParallelTopology.from_config(parallel_config, world_size=runtime.world_size)
        plan = DEFAULT_GROUP_PLAN if group_plan is None else group_plan
        _validate_plan(plan)
        registry = ParallelGroupRegistry(runtime, topology).materialize(plan)
        return cls(topology=topology, registry=registry, rank=runtime.rank,
                   sequence_parallel=parallel_config.sequence_parallel)

    rank = property(lambda self: self._rank)
    world_size = property(lambda self: self.topology.world_size)
    sequence_parallel = property(lambda self: self._sequence_parallel)

    def group(self, key: GroupKeyLike) -> ParallelGroup:
        return self.registry.group(key)

    def has_group(self, key: GroupKeyLike) -> bool:
        return self.registry.has_group(key)

    def axis_group(self, axis: ParallelAxis | str) -> ParallelGroup:
        return self.group(_AXIS_KEYS[ParallelAxis.parse(axis)])

    def mesh(self, key: GroupKeyLike) -> Any:
        return self.registry.mesh(key)

    def group_plan(self) -> GroupPlan:
        return self.registry.plan

    def group_family(self, key: GroupKeyLike) -> tuple[tuple[int, ...], ...]:
        return self.registry.family(key)

    tp = property(lambda self: self.group(GroupKey.TP))
    pp = property(lambda self: self.group(GroupKey.PP))
    cp = property(lambda self: self.group(GroupKey.CP))
    ep = property(lambda self: self.group(GroupKey.EP))
    dp = property(lambda self: self.group(GroupKey.DP_AXIS))
    dense_replica = property(lambda self: self.group(GroupKey.DENSE_REPLICA))
    expert_replica = property(lambda self: self.group(GroupKey.EXPERT_REPLICA))
    batch_replica = property(lambda self: self.group(GroupKey.BATCH_REPLICA))

    def is_pipeline_first_stage(self) -> bool:
        return self.coordinate.pp == 0

    def is_pipeline_last_stage(self) -> bool:
        return self.coordinate.pp == self.topology.pipeline_parallel_size - 1

    def pipeline_prev_rank(self) -> int | None:
        if self.is_pipeline_first_stage():
            return None
        return self.pp.global_rank_at(self.coordinate.pp - 1)

    def pipeline_next_rank(self) -> int | None:
        if self.is_pipeline_last_stage():
            return None
        return self.pp.global_rank_at(self.coordinate.pp + 1)

    def close(self) -> None:
        self.registry.close()

    def __enter__(self) -> "ParallelContext":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __repr__(self) -> str:
        return f"ParallelContext(rank={self.rank}, coordinate={self.coordinate}, {self.topology!r})"


def _validate_plan(plan: GroupPlan) -> None:
    """A custom plan may add families but not redefine the built-in ones."""
    for key in GroupKey:
        try:
            spec = plan.spec(key)
        except KeyError:
            raise ValueError(f"group plan must define built-in group {key.value!r}") from None
        builtin = DEFAULT_GROUP_PLAN.spec(key)
        if (spec.varying_axes, dict(spec.select), spec.channel) != (
                builtin.varying_axes, dict(builtin.select), builtin.channel):
            raise ValueError(f"group plan redefines built-in group {key.value!r}")
