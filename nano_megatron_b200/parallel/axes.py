"""The five parallel axes, per-rank coordinates, and rank-order parsing.

Reference behaviour: src/nano_megatron/parallel/axes.py:16-120. Coordinates are
always listed in the semantic order (tp, cp, ep, dp, pp); the *rank order* is a
separate permutation whose left-most axis varies fastest. Torch-free so that
configuration and checkpoint tooling can use it without a device.
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator, Mapping
from dataclasses import dataclass
from enum import StrEnum


class ParallelAxis(StrEnum):
    TP = "tp"
    PP = "pp"
    CP = "cp"
    EP = "ep"
    DP = "dp"

    @classmethod
    def parse(cls, value: "ParallelAxis | str") -> "ParallelAxis":
        if isinstance(value, cls):
            return value
        text = str(value).strip().lower()
        for axis in cls:
            if axis.value == text:
                return axis
        names = ", ".join(a.value for a in cls)
        raise ValueError(f"unknown parallel axis {value!r}; expected one of: {names}")


PARALLEL_AXES: tuple[ParallelAxis, ...] = (
    ParallelAxis.TP,
    ParallelAxis.CP,
    ParallelAxis.EP,
    ParallelAxis.DP,
    ParallelAxis.PP,
)
DEFAULT_RANK_ORDER: tuple[ParallelAxis, ...] = PARALLEL_AXES


@dataclass(frozen=True, slots=True)
class ParallelCoordinate:
    """One rank's position along each axis (field order tp, cp, ep, dp, pp)."""

    tp: int
    cp: int
    ep: int
    dp: int
    pp: int

    def get(self, axis: ParallelAxis | str) -> int:
        return getattr(self, ParallelAxis.parse(axis).value)

    def __getitem__(self, axis: ParallelAxis | str) -> int:
        return self.get(axis)

    def __iter__(self) -> Iterator[int]:
        return iter((self.tp, self.cp, self.ep, self.dp, self.pp))

    def as_dict(self) -> dict[ParallelAxis, int]:
        return {axis: self.get(axis) for axis in PARALLEL_AXES}

    def replace(self, **changes: int) -> "ParallelCoordinate":
        allowed = {a.value for a in PARALLEL_AXES}
        bad = sorted(set(changes) - allowed)
        if bad:
            raise TypeError(f"unknown coordinate field(s): {', '.join(bad)}")
        values = {a.value: self.get(a) for a in PARALLEL_AXES}
        values.update(changes)
        return ParallelCoordinate(**values)


def normalize_rank_order(order: Iterable[ParallelAxis | str]) -> tuple[ParallelAxis, ...]:
    """Parse a rank order; it must name each of the five axes exactly once."""
    parsed = tuple(ParallelAxis.parse(a) for a in order)
    seen = set(parsed)
    if len(parsed) == len(PARALLEL_AXES) and seen == set(PARALLEL_AXES):
        return parsed
    problems = []
    missing = sorted(a.value for a in set(PARALLEL_AXES) - seen)
    dupes = sorted({a.value for a in parsed if parsed.count(a) > 1})
    if missing:
        problems.append(f"missing={missing}")
    if dupes:
        problems.append(f"duplicates={dupes}")
    if not problems:
        problems.append(f"received {len(parsed)} entries")
    raise ValueError(
        "rank order must contain tp, pp, cp, ep, and dp exactly once (" + "; ".join(problems) + ")"
    )


def coordinate_mapping(values: Mapping[ParallelAxis | str, int]) -> dict[ParallelAxis, int]:
    out: dict[ParallelAxis, int] = {}
    for raw, v in values.items():
        axis = ParallelAxis.parse(raw)
        if axis in out:
            raise ValueError(f"coordinate for axis {axis.value!r} was specified twice")
        out[axis] = v
    missing = sorted(a.value for a in set(PARALLEL_AXES) - set(out))
    if missing:
        raise ValueError(f"coordinate is missing axis value(s): {', '.join(missing)}")
    return out
