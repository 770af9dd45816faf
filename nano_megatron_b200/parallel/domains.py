"""Parameter domains: which replica group reduces each parameter's gradient.

Dense parameters reduce over DENSE_REPLICA (dp x ep x cp); expert parameters
over EXPERT_REPLICA (dp x cp). Registration is by identity and never mutates
the parameter. Reference: src/nano_megatron/parallel/domains.py:13-243.
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator
from dataclasses import dataclass
from enum import StrEnum
from typing import Any

from .group_plan import GroupKey, GroupKeyLike, normalize_group_key


class ParameterDomain(StrEnum):
    DENSE = "dense"
    EXPERT = "expert"

    @classmethod
    def parse(cls, value: "ParameterDomain | str") -> "ParameterDomain":
        if isinstance(value, cls):
            return value
        try:
            return cls(str(value).strip().lower())
        except ValueError as error:
            raise ValueError(f"unknown parameter domain {value!r}") from error


_DEFAULT_REPLICA = {ParameterDomain.DENSE: GroupKey.DENSE_REPLICA,
                    ParameterDomain.EXPERT: GroupKey.EXPERT_REPLICA}


def default_replica_group(domain: ParameterDomain | str) -> GroupKey:
    return _DEFAULT_REPLICA[ParameterDomain.parse(domain)]


@dataclass(frozen=True, slots=True)
class ParameterPlacement:
    domain: ParameterDomain
    tensor_sharded: bool
    replica_group: GroupKeyLike
    tensor_shard_dim: int | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "domain", ParameterDomain.parse(self.domain))
        object.__setattr__(self, "replica_group", normalize_group_key(self.replica_group))
        if not isinstance(self.tensor_sharded, bool):
            raise TypeError("tensor_sharded must be a boolean")
        d = self.tensor_shard_dim
        if d is not None:
            if isinstance(d, bool) or not isinstance(d, int) or d < 0:
                raise ValueError("tensor_shard_dim must be a non-negative integer or null")
            if not self.tensor_sharded:
                raise ValueError("tensor_shard_dim requires tensor_sharded=True")

    @classmethod
    def for_domain(cls, domain, *, tensor_sharded: bool = False,
                   replica_group: GroupKeyLike | None = None,
                   tensor_shard_dim: int | None = None) -> "ParameterPlacement":
        d = ParameterDomain.parse(domain)
        return cls(d, tensor_sharded, _DEFAULT_REPLICA[d] if replica_group is None
                   else replica_group, tensor_shard_dim)


class ParameterDomainRegistry:
    def __init__(self) -> None:
        self._entries: dict[int, list] = {}  # id -> [param, placement, name]

    def register(self, parameter: Any, placement=None, *, domain=None, tensor_sharded=False,
                 replica_group=None, tensor_shard_dim=None, name: str | None = None
                 ) -> ParameterPlacement:
        if parameter is None:
            raise TypeError("cannot register None as a parameter")
        if isinstance(placement, ParameterPlacement):
            if domain is not None or tensor_sharded or replica_group is not None \
                    or tensor_shard_dim is not None:
                raise ValueError("domain/tensor_sharded/replica_group cannot accompany an "
                                 "explicit placement")
            resolved = placement
        else:
            if placement is not None and domain is not None:
                raise ValueError("parameter domain was supplied both positionally and by keyword")
            resolved = ParameterPlacement.for_domain(
                domain or placement or ParameterDomain.DENSE, tensor_sharded=tensor_sharded,
                replica_group=replica_group, tensor_shard_dim=tensor_shard_dim)
        entry = self._entries.get(id(parameter))
        if entry is not None:
            if entry[0] is not parameter:
                raise RuntimeError("parameter identity collision in domain registry")
            if entry[1] != resolved:
                raise ValueError(f"parameter is already registered with {entry[1]}, "
                                 f"cannot use {resolved}")
            if name is not None and entry[2] not in (None, name):
                raise ValueError(f"parameter is already registered as {entry[2]!r}, "
                                 f"cannot rename to {name!r}")
            entry[2] = entry[2] or name
            return entry[1]
        self._entries[id(parameter)] = [parameter, resolved, name]
        return resolved

    def register_module(self, module: Any, placement=None, *, prefix: str = "", **kwargs
                        ) -> None:
        for pname, p in module.named_parameters():
            self.register(p, placement, name=f"{prefix}{pname}", **kwargs)

    def unregister(self, parameter: Any) -> None:
        self._entries.pop(id(parameter), None)

    def _entry(self, parameter: Any) -> list:
        entry = self._entries.get(id(parameter))
        if entry is None or entry[0] is not parameter:
            raise KeyError("parameter is not registered in the domain registry")
        return entry

    def placement(self, parameter: Any) -> ParameterPlacement:
        return self._entry(parameter)[1]

    def get(self, parameter: Any, default: Any = None):
        entry = self._entries.get(id(parameter))
        return default if entry is None or entry[0] is not parameter else entry[1]

    def domain(self, parameter: Any) -> ParameterDomain:
        return self.placement(parameter).domain

    def replica_group(self, parameter: Any) -> GroupKeyLike:
        return self.placement(parameter).replica_group

    def name(self, parameter: Any) -> str | None:
        return self._entry(parameter)[2]

    def parameters(self, domain=None) -> tuple[Any, ...]:
        d = None if domain is None else ParameterDomain.parse(domain)
        return tuple(e[0] for e in self._entries.values() if d is None or e[1].domain is d)

    def grouped_parameters(self) -> dict[ParameterDomain, tuple[Any, ...]]:
        return {d: self.parameters(d) for d in ParameterDomain if self.parameters(d)}

    def items(self) -> Iterator[tuple[Any, ParameterPlacement]]:
        return ((e[0], e[1]) for e in self._entries.values())

    def validate_complete(self, parameters: Iterable[Any]) -> None:
        missing = [p for p in parameters if id(p) not in self._entries]
        if missing:
            raise ValueError(f"{len(missing)} parameter(s) have no registered domain")

    def __contains__(self, parameter: object) -> bool:
        e = self._entries.get(id(parameter))
        return e is not None and e[0] is parameter

    def __len__(self) -> int:
        return len(self._entries)
