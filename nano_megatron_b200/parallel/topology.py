"""Pure rank <-> coordinate arithmetic for the five-axis topology.

Reference behaviour: src/nano_megatron/parallel/topology.py:31-235 (strides from
the rank order, left-most axis fastest; replica sizes batch = DP*EP,
dense = DP*EP*CP, expert = DP*CP).
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator, Mapping, Sequence
from types import MappingProxyType

from .axes import (
    DEFAULT_RANK_ORDER,
    PARALLEL_AXES,
    ParallelAxis,
    ParallelCoordinate,
    coordinate_mapping,
    normalize_rank_order,
)


def _check_size(axis: ParallelAxis, value: object) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"size for axis {axis.value!r} must be an integer, got {value!r}")
    if value < 1:
        raise ValueError(f"size for axis {axis.value!r} must be >= 1, got {value}")
    return value


class ParallelTopology:
    """Immutable mapping between global ranks and five-axis coordinates."""

    __slots__ = ("_sizes", "order", "_strides", "world_size")

    def __init__(self, sizes: Mapping[ParallelAxis | str, int],
                 order: Sequence[ParallelAxis | str] = DEFAULT_RANK_ORDER) -> None:
        parsed: dict[ParallelAxis, int] = {}
        for raw, value in sizes.items():
            axis = ParallelAxis.parse(raw)
            if axis in parsed:
                raise ValueError(f"size for axis {axis.value!r} was specified more than once")
            parsed[axis] = _check_size(axis, value)
        missing = sorted(a.value for a in set(PARALLEL_AXES) - set(parsed))
        if missing or len(parsed) != len(PARALLEL_AXES):
            raise ValueError(
                "sizes must define all five parallel axes; missing: " + (", ".join(missing) or "none")
            )
        norm = normalize_rank_order(order)
        strides, running = {}, 1
        for axis in norm:
            strides[axis] = running
            running *= parsed[axis]
        object.__setattr__(self, "_sizes", MappingProxyType(parsed))
        object.__setattr__(self, "order", norm)
        object.__setattr__(self, "_strides", MappingProxyType(strides))
        object.__setattr__(self, "world_size", running)

    def __setattr__(self, name, value):  # immutable
        raise AttributeError("ParallelTopology is immutable")

    def __eq__(self, other: object) -> bool:
        return (isinstance(other, ParallelTopology) and dict(self._sizes) == dict(other._sizes)
                and self.order == other.order)

    def __hash__(self) -> int:
        return hash((tuple(sorted((a.value, s) for a, s in self._sizes.items())), self.order))

    @classmethod
    def from_sizes(cls, *, tensor: int = 1, pipeline: int = 1, context: int = 1, expert: int = 1,
                   data: int = 1, order: Sequence[ParallelAxis | str] = DEFAULT_RANK_ORDER
                   ) -> "ParallelTopology":
        return cls({ParallelAxis.TP: tensor, ParallelAxis.PP: pipeline, ParallelAxis.CP: context,
                    ParallelAxis.EP: expert, ParallelAxis.DP: data}, order)

    @classmethod
    def from_config(cls, config, *, world_size: int | None = None) -> "ParallelTopology":
        return cls.from_sizes(tensor=config.tensor, pipeline=config.pipeline,
                              context=config.context, expert=config.expert,
                              data=config.resolve_data_parallel_size(world_size), order=config.order)

    @property
    def sizes(self) -> Mapping[ParallelAxis, int]:
        return self._sizes

    def size(self, axis: ParallelAxis | str) -> int:
        return self._sizes[ParallelAxis.parse(axis)]

    def stride(self, axis: ParallelAxis | str) -> int:
        return self._strides[ParallelAxis.parse(axis)]

    tensor_parallel_size = property(lambda self: self.size(ParallelAxis.TP))
    pipeline_parallel_size = property(lambda self: self.size(ParallelAxis.PP))
    context_parallel_size = property(lambda self: self.size(ParallelAxis.CP))
    expert_parallel_size = property(lambda self: self.size(ParallelAxis.EP))
    data_parallel_size = property(lambda self: self.size(ParallelAxis.DP))

    @property
    def batch_replica_size(self) -> int:
        return self.data_parallel_size * self.expert_parallel_size

    @property
    def dense_replica_size(self) -> int:
        return self.batch_replica_size * self.context_parallel_size

    @property
    def expert_replica_size(self) -> int:
        return self.data_parallel_size * self.context_parallel_size

    def rank_to_coordinate(self, rank: int) -> ParallelCoordinate:
        if isinstance(rank, bool) or not isinstance(rank, int):
            raise TypeError(f"rank must be an integer, got {rank!r}")
        if not 0 <= rank < self.world_size:
            raise ValueError(f"rank must be in [0, {self.world_size}), got {rank}")
        return ParallelCoordinate(**{
            a.value: (rank // self._strides[a]) % self._sizes[a] for a in PARALLEL_AXES
        })

    def coordinate_to_rank(self, coordinate: ParallelCoordinate | Mapping[ParallelAxis | str, int]
                           ) -> int:
        values = coordinate.as_dict() if isinstance(coordinate, ParallelCoordinate) \
            else coordinate_mapping(coordinate)
        rank = 0
        for axis in PARALLEL_AXES:
            v, n = values[axis], self._sizes[axis]
            if isinstance(v, bool) or not isinstance(v, int):
                raise TypeError(f"coordinate for axis {axis.value!r} must be an integer, got {v!r}")
            if not 0 <= v < n:
                raise ValueError(f"coordinate for axis {axis.value!r} must be in [0, {n}), got {v}")
            rank += v * self._strides[axis]
        return rank

    def iter_coordinates(self) -> Iterator[ParallelCoordinate]:
        return (self.rank_to_coordinate(r) for r in range(self.world_size))

    def ranks_varying(self, rank: int, varying_axes: Iterable[ParallelAxis | str]) -> tuple[int, ...]:
        """Ranks that share ``rank``'s coordinate on every axis not in ``varying_axes``."""
        vary = [ParallelAxis.parse(a) for a in varying_axes]
        base = self.rank_to_coordinate(rank).as_dict()
        for a in vary:
            base[a] = 0
        start = self.coordinate_to_rank(base)
        ranks = [start]
        for a in vary:
            step = self._strides[a]
            ranks = [r + i * step for r in ranks for i in range(self._sizes[a])]
        return tuple(sorted(ranks))

    def __len__(self) -> int:
        return self.world_size

    def __repr__(self) -> str:
        sizes = ", ".join(f"{a.value}={self.size(a)}" for a in PARALLEL_AXES)
        return f"ParallelTopology({sizes}, order={'-'.join(a.value for a in self.order)!r})"
