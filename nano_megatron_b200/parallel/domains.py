"""Parameter domains: which replica group sums each parameter's gradient.

A parameter is either *dense* (identical on every data / expert / context replica: its
gradient is summed over DENSE_REPLICA = dp x ep x cp) or *expert* (different per EP
rank: summed over EXPERT_REPLICA = dp x cp). A :class:`ParameterPlacement` records the
domain, the replica group and whether (and along which dim) the tensor is split over TP;
the data-parallel buffers cut their buckets per domain and the checkpoint mapping uses the
shard dim. The registry is keyed by object identity, holds a strong reference to each
parameter and never modifies one. The public names and the two default groups are the
reference's (src/nano_megatron/parallel/domains.py).
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
        known = {d.value: d for d in cls}
        if isinstance(value, str) and value.strip().lower() in known:
            return known[value.strip().lower()]
        raise ValueError(f"{value!r} names no parameter domain (known: {', '.join(known)})")


_REPLICA_OF = {ParameterDomain.DENSE: GroupKey.DENSE_REPLICA,
               ParameterDomain.EXPERT: GroupKey.EXPERT_REPLICA}


def default_replica_group(domain: ParameterDomain | str) -> GroupKey:
    """The group a domain's gradients are summed over unless a placement says otherwise."""
    return _REPLICA_OF[ParameterDomain.parse(domain)]


@dataclass(frozen=True, slots=True)
class ParameterPlacement:
    domain: ParameterDomain
    tensor_sharded: bool
    replica_group: GroupKeyLike
    tensor_shard_dim: int | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "domain", ParameterDomain.parse(self.domain))
        object.__setattr__(self, "replica_group", normalize_group_key(self.replica_group))
        if type(self.tensor_sharded) is not bool:
            raise TypeError(f"tensor_sharded is {self.tensor_sharded!r}, not a bool")
        dim = self.tensor_shard_dim
        if dim is None:
            return
        if type(dim) is not int or dim < 0:
            raise ValueError(f"tensor_shard_dim {dim!r} is not a dimension index (int >= 0)")
        if not self.tensor_sharded:
            raise ValueError(f"tensor_shard_dim={dim} given for a tensor that is not "
                             "sharded over TP (set tensor_sharded=True)")

    @classmethod
    def for_domain(cls, domain, *, tensor_sharded: bool = False,
                   replica_group: GroupKeyLike | None = None,
                   tensor_shard_dim: int | None = None) -> "ParameterPlacement":
        d = ParameterDomain.parse(domain)
        group = _REPLICA_OF[d] if replica_group is None else replica_group
        return cls(d, tensor_sharded, group, tensor_shard_dim)


def _resolve(placement, domain, tensor_sharded, replica_group,
             tensor_shard_dim) -> ParameterPlacement:
    """One placement from ``register``'s arguments: an explicit placement object, or a
    domain (positional or keyword, default dense) plus the placement fields."""
    if isinstance(placement, ParameterPlacement):
        extras = {"domain": domain is not None, "tensor_sharded": bool(tensor_sharded),
                  "replica_group": replica_group is not None,
                  "tensor_shard_dim": tensor_shard_dim is not None}
        given = [k for k, v in extras.items() if v]
        if given:
            raise ValueError("an explicit ParameterPlacement already fixes " +
                             ", ".join(given) + "; pass one or the other")
        return placement
    if placement is not None and domain is not None:
        raise ValueError(f"domain given twice ({placement!r} positionally, {domain!r} by "
                         "keyword)")
    chosen = placement if placement is not None else domain
    return ParameterPlacement.for_domain(
        ParameterDomain.DENSE if chosen is None else chosen, tensor_sharded=tensor_sharded,
        replica_group=replica_group, tensor_shard_dim=tensor_shard_dim)


class _Entry:
    __slots__ = ("param", "placement", "name")

    def __init__(self, param, placement, name) -> None:
        self.param, self.placement, self.name = param, placement, name


class ParameterDomainRegistry:
    """Placement of every model parameter, looked up by identity."""

    def __init__(self) -> None:
        self._by_id: dict[int, _Entry] = {}

    def _find(self, parameter: Any) -> _Entry | None:
        e = self._by_id.get(id(parameter))
        return e if e is not None and e.param is parameter else None

    def _need(self, parameter: Any) -> _Entry:
        e = self._find(parameter)
        if e is None:
            raise KeyError(f"parameter of shape {tuple(getattr(parameter, 'shape', ()))} has "
                           "no placement in this registry")
        return e

    # ------------------------------------------------------------------ registration
    def register(self, parameter: Any, placement=None, *, domain=None, tensor_sharded=False,
                 replica_group=None, tensor_shard_dim=None, name: str | None = None
                 ) -> ParameterPlacement:
        """Record a parameter's placement. Registering it again is a no-op if the
        placement agrees (a name may be added later, not changed); a different placement
        is an error: one tensor has one gradient reduction."""
        if parameter is None:
            raise TypeError("register() got None instead of a parameter")
        want = _resolve(placement, domain, tensor_sharded, replica_group, tensor_shard_dim)
        old = self._by_id.get(id(parameter))
        if old is None:
            self._by_id[id(parameter)] = _Entry(parameter, want, name)
            return want
        if old.param is not parameter:     # only if an entry outlived its object's id
            raise RuntimeError("stale registry entry shares this parameter's id")
        label = old.name or name or "parameter"
        if old.placement != want:
            raise ValueError(f"{label} is already registered as {old.placement}; "
                             f"refusing {want}")
        if name is not None and old.name is not None and old.name != name:
            raise ValueError(f"cannot rename {old.name!r} to {name!r}")
        if old.name is None:
            old.name = name
        return old.placement

    def register_module(self, module: Any, placement=None, *, prefix: str = "", **kwargs
                        ) -> None:
        """Register every parameter of ``module`` under ``prefix + its dotted name``."""
        for pname, p in module.named_parameters():
            self.register(p, placement, name=prefix + pname, **kwargs)

    def unregister(self, parameter: Any) -> None:
        if self._find(parameter) is not None:
            del self._by_id[id(parameter)]

    # ------------------------------------------------------------------ queries
    def placement(self, parameter: Any) -> ParameterPlacement:
        return self._need(parameter).placement

    def get(self, parameter: Any, default: Any = None):
        e = self._find(parameter)
        return default if e is None else e.placement

    def domain(self, parameter: Any) -> ParameterDomain:
        return self._need(parameter).placement.domain

    def replica_group(self, parameter: Any) -> GroupKeyLike:
        return self._need(parameter).placement.replica_group

    def name(self, parameter: Any) -> str | None:
        return self._need(parameter).name

    def parameters(self, domain=None) -> tuple[Any, ...]:
        keep = None if domain is None else ParameterDomain.parse(domain)
        return tuple(e.param for e in self._by_id.values()
                     if keep is None or e.placement.domain is keep)

    def grouped_parameters(self) -> dict[ParameterDomain, tuple[Any, ...]]:
        out: dict[ParameterDomain, list] = {}
        for e in self._by_id.values():
            out.setdefault(e.placement.domain, []).append(e.param)
        return {d: tuple(out[d]) for d in ParameterDomain if d in out}

    def items(self) -> Iterator[tuple[Any, ParameterPlacement]]:
        return iter([(e.param, e.placement) for e in self._by_id.values()])

    def validate_complete(self, parameters: Iterable[Any]) -> None:
        """Every given parameter must have a placement (the DP buffers need one each)."""
        count = sum(1 for p in parameters if self._find(p) is None)
        if count:
            raise ValueError(f"{count} parameter(s) have no registered domain")

    def __contains__(self, parameter: object) -> bool:
        return self._find(parameter) is not None

    def __len__(self) -> int:
        return len(self._by_id)
