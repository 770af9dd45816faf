"""Parallel topology, process groups, RNG streams and parameter domains."""

from .axes import DEFAULT_RANK_ORDER, PARALLEL_AXES, ParallelAxis, ParallelCoordinate, normalize_rank_order
from .context import ParallelContext
from .domains import ParameterDomain, ParameterDomainRegistry, ParameterPlacement, default_replica_group
from .group import LocalGroup, ParallelGroup, require_parallel_group
from .group_plan import DEFAULT_GROUP_PLAN, GroupKey, GroupKeyLike, GroupPlan, GroupSpec, PlannedGroup
from .layout import TensorLayout
from .registry import GroupRegistry, ParallelGroupRegistry
from .rng import ParallelRNG, RNGStream
from .topology import ParallelTopology

__all__ = [n for n in dir() if not n.startswith("_")]
