"""Declarative process-group families over the five-axis topology.

A :class:`GroupSpec` names the axes that vary *inside* one group; every
combination of the remaining axes yields a separate group. ``select``
restricts coordinates (negative indices count from the end), ``channel`` lets
several communicators cover the same ranks. The default plan has the same 13
families as the reference (src/nano_megatron/parallel/group_plan.py:206-246),
including two extra pipeline transport channels and the first/last-stage
EMBEDDING group.
"""

from __future__ import annotations

from collections.abc import Iterator, Mapping
from dataclasses import dataclass, field
from enum import StrEnum
from types import MappingProxyType

from .axes import PARALLEL_AXES, ParallelAxis
from .topology import ParallelTopology


class GroupKey(StrEnum):
    TP = "tp"
    PP = "pp"
    PP_TRANSPORT_1 = "pp_transport_1"
    PP_TRANSPORT_2 = "pp_transport_2"
    CP = "cp"
    EP = "ep"
    DP_AXIS = "dp_axis"
    TP_CP = "tp_cp"
    TP_EP = "tp_ep"
    DENSE_REPLICA = "dense_replica"
    EXPERT_REPLICA = "expert_replica"
    BATCH_REPLICA = "batch_replica"
    EMBEDDING = "embedding"


GroupKeyLike = GroupKey | str


def normalize_group_key(key: GroupKeyLike) -> GroupKeyLike:
    if isinstance(key, GroupKey):
        return key
    if not isinstance(key, str) or not key.strip():
        raise TypeError(f"group key must be a GroupKey or non-empty string, got {key!r}")
    text = key.strip()
    return GroupKey(text) if text in GroupKey._value2member_map_ else text


@dataclass(frozen=True, slots=True)
class GroupSpec:
    key: GroupKeyLike
    varying_axes: frozenset
    select: Mapping = field(default_factory=dict)
    backend: str | None = None
    channel: str = "default"

    def __post_init__(self) -> None:
        axes = frozenset(ParallelAxis.parse(a) for a in self.varying_axes)
        if not axes:
            raise ValueError("a group spec must vary at least one parallel axis")
        sel: dict[ParallelAxis, tuple[int, ...]] = {}
        for raw, idx in dict(self.select).items():
            axis = ParallelAxis.parse(raw)
            if axis in sel:
                raise ValueError(f"selection for axis {axis.value!r} was specified twice")
            idx = tuple(idx)
            if not idx:
                raise ValueError(f"selection for axis {axis.value!r} cannot be empty")
            if any(isinstance(i, bool) or not isinstance(i, int) for i in idx):
                raise TypeError(f"selection for axis {axis.value!r} must contain integers")
            sel[axis] = idx
        if self.backend is not None and not self.backend.strip():
            raise ValueError("group backend cannot be an empty string")
        if not isinstance(self.channel, str) or not self.channel.strip():
            raise ValueError("group channel must be a non-empty string")
        object.__setattr__(self, "key", normalize_group_key(self.key))
        object.__setattr__(self, "varying_axes", axes)
        object.__setattr__(self, "select", MappingProxyType(sel))
        object.__setattr__(self, "backend", self.backend.strip() if self.backend else None)
        object.__setattr__(self, "channel", self.channel.strip())


@dataclass(frozen=True, slots=True)
class PlannedGroup:
    spec: GroupSpec
    ranks: tuple[int, ...]
    fixed_coordinate: Mapping

    key = property(lambda self: self.spec.key)
    backend = property(lambda self: self.spec.backend)
    channel = property(lambda self: self.spec.channel)


def _resolve_selection(size: int, selection: tuple[int, ...] | None) -> tuple[int, ...]:
    if selection is None:
        return tuple(range(size))
    out: list[int] = []
    for raw in selection:
        i = raw + size if raw < 0 else raw
        if not 0 <= i < size:
            raise ValueError(f"group selection index {raw} is out of range for axis size {size}")
        if i not in out:
            out.append(i)
    return tuple(out)


class GroupPlan:
    """Ordered, uniquely keyed collection of group specs."""

    __slots__ = ("specs",)

    def __init__(self, *specs) -> None:
        if len(specs) == 1 and not isinstance(specs[0], GroupSpec):
            specs = tuple(specs[0])
        if any(not isinstance(s, GroupSpec) for s in specs):
            raise TypeError("GroupPlan entries must be GroupSpec instances")
        keys = [s.key for s in specs]
        for k in keys:
            if keys.count(k) > 1:
                raise ValueError(f"group key {k!s} is declared more than once")
        self.specs = tuple(specs)

    def spec(self, key: GroupKeyLike) -> GroupSpec:
        k = normalize_group_key(key)
        for s in self.specs:
            if s.key == k:
                return s
        raise KeyError(f"group key {k!s} is not present in this plan")

    def extend(self, *specs: GroupSpec) -> "GroupPlan":
        return GroupPlan(*self.specs, *specs)

    def expand(self, topology: ParallelTopology) -> tuple[PlannedGroup, ...]:
        return tuple(g for s in self.specs for g in self.expand_spec(topology, s))

    def groups(self, topology: ParallelTopology, key: GroupKeyLike) -> tuple[PlannedGroup, ...]:
        return self.expand_spec(topology, self.spec(key))

    @staticmethod
    def expand_spec(topology: ParallelTopology, spec: GroupSpec) -> tuple[PlannedGroup, ...]:
        allowed = {a: set(_resolve_selection(topology.size(a), spec.select.get(a)))
                   for a in PARALLEL_AXES}
        fixed_axes = tuple(a for a in topology.order if a not in spec.varying_axes)
        buckets: dict[tuple[int, ...], list[int]] = {}
        for rank in range(topology.world_size):
            c = topology.rank_to_coordinate(rank)
            if all(c.get(a) in allowed[a] for a in PARALLEL_AXES):
                buckets.setdefault(tuple(c.get(a) for a in fixed_axes), []).append(rank)
        return tuple(PlannedGroup(spec, tuple(r), MappingProxyType(dict(zip(fixed_axes, k))))
                     for k, r in buckets.items())

    def __iter__(self) -> Iterator[GroupSpec]:
        return iter(self.specs)

    def __len__(self) -> int:
        return len(self.specs)


_A = ParallelAxis
DEFAULT_GROUP_PLAN = GroupPlan(
    GroupSpec(GroupKey.TP, frozenset({_A.TP})),
    GroupSpec(GroupKey.PP, frozenset({_A.PP})),
    # Extra pipeline communicators: a receive can be waited on without also
    # draining an in-flight send that NCCL coalesced into the same Work.
    GroupSpec(GroupKey.PP_TRANSPORT_1, frozenset({_A.PP}), channel="pp_transport_1"),
    GroupSpec(GroupKey.PP_TRANSPORT_2, frozenset({_A.PP}), channel="pp_transport_2"),
    GroupSpec(GroupKey.CP, frozenset({_A.CP})),
    GroupSpec(GroupKey.EP, frozenset({_A.EP})),
    GroupSpec(GroupKey.DP_AXIS, frozenset({_A.DP})),
    GroupSpec(GroupKey.TP_CP, frozenset({_A.TP, _A.CP})),
    GroupSpec(GroupKey.TP_EP, frozenset({_A.TP, _A.EP})),
    GroupSpec(GroupKey.DENSE_REPLICA, frozenset({_A.DP, _A.EP, _A.CP})),
    GroupSpec(GroupKey.EXPERT_REPLICA, frozenset({_A.DP, _A.CP})),
    GroupSpec(GroupKey.BATCH_REPLICA, frozenset({_A.TP, _A.PP, _A.CP})),
    GroupSpec(GroupKey.EMBEDDING, frozenset({_A.PP}), select={_A.PP: (0, -1)}),
)
