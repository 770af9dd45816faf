"""One materialised process group as seen by the local rank.

Reference: src/nano_megatron/parallel/group.py:11-75.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from .group_plan import GroupKeyLike


@dataclass(frozen=True, slots=True)
class ParallelGroup:
    key: GroupKeyLike
    ranks: tuple[int, ...]
    process_group: Any | None
    rank: int
    size: int
    backend: str
    channel: str = "default"

    def __post_init__(self) -> None:
        if not self.ranks:
            raise ValueError("parallel group ranks cannot be empty")
        if len(set(self.ranks)) != len(self.ranks):
            raise ValueError("parallel group ranks cannot contain duplicates")
        if tuple(sorted(self.ranks)) != tuple(self.ranks):
            raise ValueError("parallel group ranks must be sorted")
        if self.size != len(self.ranks):
            raise ValueError(f"group size {self.size} does not match {len(self.ranks)} ranks")
        if not 0 <= self.rank < self.size:
            raise ValueError(f"local group rank must be in [0, {self.size}), got {self.rank}")
        if self.size > 1 and self.process_group is None:
            raise ValueError("a multi-rank ParallelGroup requires a materialized process_group")

    @property
    def global_rank(self) -> int:
        return self.ranks[self.rank]

    @property
    def is_distributed(self) -> bool:
        return self.size > 1

    def contains(self, global_rank: int) -> bool:
        return global_rank in self.ranks

    def global_rank_at(self, group_rank: int) -> int:
        if not 0 <= group_rank < self.size:
            raise ValueError(f"group rank must be in [0, {self.size}), got {group_rank}")
        return self.ranks[group_rank]


def require_parallel_group(group: Any, *, name: str) -> Any:
    """Check that ``group`` quacks like a ParallelGroup (rank/size/ranks/process_group)."""
    for attr in ("rank", "size", "ranks", "process_group"):
        if not hasattr(group, attr):
            raise TypeError(f"{name} must be a ParallelGroup-like object (missing {attr!r})")
    if group.size > 1 and group.process_group is None:
        raise ValueError(f"{name} spans {group.size} ranks but has no process group")
    return group


@dataclass(frozen=True, slots=True)
class LocalGroup:
    """A size-one group for single-process use (tests, inference, CPU smoke runs)."""

    key: GroupKeyLike = "local"
    ranks: tuple[int, ...] = (0,)
    process_group: Any | None = None
    rank: int = 0
    size: int = 1
    backend: str = "local"
    channel: str = "default"
    global_rank = property(lambda self: 0)
    is_distributed = property(lambda self: False)
