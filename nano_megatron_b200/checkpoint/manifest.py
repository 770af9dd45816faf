"""Checkpoint manifest (schema version 2) and per-tensor shard metadata.

The JSON layout is the reference's on-disk format (src/nano_megatron/checkpoint/
manifest.py:19-340 and mapping.py:13-220) so that checkpoints written here can
be read by the reference's export tool and vice versa: same field names,
shard-id scheme (``tpXXXX_ppXXXX_epXXXX``), runtime-state ids
(``tpXXXX_ppXXXX_cpXXXX_epXXXX_dpXXXX``), topology-compatibility block and
``framework = "nano-megatron"``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Mapping

import torch

from nano_megatron_b200.parallel.axes import ParallelAxis
from nano_megatron_b200.parallel.domains import ParameterDomain
from nano_megatron_b200.parallel.group_plan import GroupKey

SCHEMA_VERSION = 2
FRAMEWORK = "nano-megatron"


@dataclass(frozen=True)
class ShardMetadata:
    logical_key: str
    global_shape: tuple[int, ...]
    local_shape: tuple[int, ...]
    global_offset: tuple[int, ...]
    sharded_axes: tuple[ParallelAxis, ...]
    parameter_domain: ParameterDomain
    replica_coordinate: tuple[int, ...]

    def __post_init__(self) -> None:
        n = len(self.global_shape)
        if len(self.local_shape) != n or len(self.global_offset) != n:
            raise ValueError("global_shape, local_shape, and global_offset must have equal rank")
        if any(s < 0 for s in (*self.global_shape, *self.local_shape)):
            raise ValueError("tensor shapes cannot contain negative values")
        for off, loc, glob in zip(self.global_offset, self.local_shape, self.global_shape):
            if off < 0 or off + loc > glob:
                raise ValueError(f"local shard [{off}, {off + loc}) exceeds global size {glob}")

    def to_dict(self) -> dict[str, Any]:
        return {"logical_key": self.logical_key, "global_shape": list(self.global_shape),
                "local_shape": list(self.local_shape), "global_offset": list(self.global_offset),
                "sharded_axes": [a.value for a in self.sharded_axes],
                "parameter_domain": self.parameter_domain.value,
                "replica_coordinate": list(self.replica_coordinate)}

    @classmethod
    def from_dict(cls, v: Mapping[str, Any]) -> "ShardMetadata":
        return cls(str(v["logical_key"]), tuple(int(x) for x in v["global_shape"]),
                   tuple(int(x) for x in v["local_shape"]),
                   tuple(int(x) for x in v["global_offset"]),
                   tuple(ParallelAxis(x) for x in v["sharded_axes"]),
                   ParameterDomain(v["parameter_domain"]),
                   tuple(int(x) for x in v["replica_coordinate"]))


def _coord(d: Mapping[str, Any]) -> dict[str, int]:
    return {k: int(d[k]) for k in ("tp", "pp", "ep", "cp", "dp")}


@dataclass(frozen=True)
class RankLocalShard:
    shard_id: str
    writer_rank: int
    tp: int
    pp: int
    ep: int
    cp: int
    dp: int
    state_file: str
    tensor_metadata: dict = field(default_factory=dict)
    layer_start: int | None = None
    layer_end: int | None = None
    layer_ranges: tuple = ()

    def to_dict(self) -> dict[str, Any]:
        return {"shard_id": self.shard_id, "writer_rank": self.writer_rank,
                "coordinate": {"tp": self.tp, "pp": self.pp, "ep": self.ep, "cp": self.cp,
                               "dp": self.dp},
                "state_file": self.state_file,
                "layer_range": None if self.layer_start is None or self.layer_end is None
                else [self.layer_start, self.layer_end],
                "layer_ranges": [list(r) for r in self.layer_ranges],
                "tensor_metadata": {k: m.to_dict() for k, m in self.tensor_metadata.items()}}

    @classmethod
    def from_dict(cls, v: Mapping[str, Any]) -> "RankLocalShard":
        c = _coord(v["coordinate"])
        lr = v.get("layer_range")
        raw = v.get("layer_ranges")
        ranges = tuple((int(a), int(b)) for a, b in raw) if raw is not None else \
            (() if lr is None else ((int(lr[0]), int(lr[1])),))
        return cls(str(v["shard_id"]), int(v["writer_rank"]), c["tp"], c["pp"], c["ep"], c["cp"],
                   c["dp"], str(v["state_file"]),
                   {str(k): ShardMetadata.from_dict(m)
                    for k, m in v.get("tensor_metadata", {}).items()},
                   None if lr is None else int(lr[0]), None if lr is None else int(lr[1]), ranges)


@dataclass(frozen=True)
class RankRuntimeState:
    state_id: str
    writer_rank: int
    tp: int
    pp: int
    cp: int
    ep: int
    dp: int
    state_file: str

    def to_dict(self) -> dict[str, Any]:
        return {"state_id": self.state_id, "writer_rank": self.writer_rank,
                "coordinate": {"tp": self.tp, "pp": self.pp, "cp": self.cp, "ep": self.ep,
                               "dp": self.dp},
                "state_file": self.state_file}

    @classmethod
    def from_dict(cls, v: Mapping[str, Any]) -> "RankRuntimeState":
        c = _coord(v["coordinate"])
        return cls(str(v["state_id"]), int(v["writer_rank"]), c["tp"], c["pp"], c["cp"], c["ep"],
                   c["dp"], str(v["state_file"]))


def json_compatible(value: Any) -> Any:
    """Convert configs (dataclasses, enums, paths, tuples) to JSON values."""
    from dataclasses import fields, is_dataclass

    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    if isinstance(value, Enum):
        return value.value
    if isinstance(value, Path):
        return str(value)
    if is_dataclass(value) and not isinstance(value, type):
        return {f.name: json_compatible(getattr(value, f.name)) for f in fields(value)}
    if isinstance(value, Mapping):
        return {str(k): json_compatible(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [json_compatible(v) for v in value]
    if hasattr(value, "specs"):  # GroupPlan
        return [{"key": str(getattr(s.key, "value", s.key)),
                 "varying_axes": sorted(a.value for a in s.varying_axes),
                 "select": {a.value: list(i) for a, i in s.select.items()},
                 "backend": s.backend, "channel": s.channel} for s in value.specs]
    return str(value)


@dataclass(frozen=True)
class CheckpointManifest:
    schema_version: int
    framework: str
    torch_version: str
    step: int
    storage_backend: str
    parallel_sizes: dict
    rank_order: tuple
    tensor_metadata: dict
    data_parallel_mode: str = "unknown"
    rank_local_shards: tuple = ()
    rank_runtime_states: tuple = ()
    topology_compatibility: Any = None
    run_config: Any = None
    group_plan: Any = None
    virtual_stages_per_rank: int = 1

    def to_dict(self) -> dict[str, Any]:
        return {"schema_version": self.schema_version, "framework": self.framework,
                "torch_version": self.torch_version, "step": self.step,
                "storage_backend": self.storage_backend, "parallel_sizes": self.parallel_sizes,
                "rank_order": list(self.rank_order),
                "tensor_metadata": {k: m.to_dict() for k, m in self.tensor_metadata.items()},
                "data_parallel_mode": self.data_parallel_mode,
                "rank_local_shards": [s.to_dict() for s in self.rank_local_shards],
                "rank_runtime_states": [s.to_dict() for s in self.rank_runtime_states],
                "topology_compatibility": json_compatible(self.topology_compatibility),
                "run_config": json_compatible(self.run_config),
                "group_plan": json_compatible(self.group_plan),
                "virtual_stages_per_rank": self.virtual_stages_per_rank}

    @classmethod
    def from_dict(cls, v: Mapping[str, Any]) -> "CheckpointManifest":
        return cls(int(v["schema_version"]), str(v["framework"]), str(v["torch_version"]),
                   int(v["step"]), str(v["storage_backend"]),
                   {str(k): int(s) for k, s in v["parallel_sizes"].items()},
                   tuple(str(x) for x in v.get("rank_order", ())),
                   {str(k): ShardMetadata.from_dict(m)
                    for k, m in v.get("tensor_metadata", {}).items()},
                   str(v.get("data_parallel_mode", "unknown")),
                   tuple(RankLocalShard.from_dict(s) for s in v.get("rank_local_shards", ())),
                   tuple(RankRuntimeState.from_dict(s) for s in v.get("rank_runtime_states", ())),
                   v.get("topology_compatibility"), v.get("run_config"), v.get("group_plan"),
                   int(v.get("virtual_stages_per_rank", 1)))

    def write(self, path: Path) -> None:
        path.write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True) + "\n")

    @classmethod
    def read(cls, path: Path) -> "CheckpointManifest":
        return cls.from_dict(json.loads(Path(path).read_text()))


_AXIS_GROUPS = {ParallelAxis.TP: GroupKey.TP, ParallelAxis.PP: GroupKey.PP,
                ParallelAxis.CP: GroupKey.CP, ParallelAxis.EP: GroupKey.EP,
                ParallelAxis.DP: GroupKey.DP_AXIS}


def parallel_sizes(parallel) -> dict[str, int]:
    return {a.value: int(parallel.group(k).size) for a, k in _AXIS_GROUPS.items()}


def parallel_rank_order(parallel) -> tuple[str, ...]:
    order = getattr(getattr(parallel, "topology", None), "order", ())
    return tuple(str(getattr(a, "value", a)) for a in order)


def make_manifest(*, step: int, storage_backend: str, parallel, metadata: Mapping,
                  data_parallel_mode: str = "unknown", rank_local_shards: tuple = (),
                  rank_runtime_states: tuple = (), run_config=None,
                  virtual_stages_per_rank: int = 1) -> CheckpointManifest:
    plan_fn = getattr(parallel, "group_plan", None)
    plan = plan_fn() if callable(plan_fn) else None
    all_meta = list(metadata.values()) + [m for s in rank_local_shards
                                         for m in s.tensor_metadata.values()]
    has_expert = any(m.parameter_domain is ParameterDomain.EXPERT for m in all_meta)
    fixed, resizable = ["tp", "pp", "cp"], ["dp"]
    if not has_expert:
        resizable.append("ep")
    if data_parallel_mode == "zero3":
        fixed, resizable = ["tp", "pp", "cp", "ep"], ["dp"]
    dcp = storage_backend == "fsdp2_dcp"
    return CheckpointManifest(
        SCHEMA_VERSION, FRAMEWORK, torch.__version__, step, storage_backend,
        parallel_sizes(parallel), parallel_rank_order(parallel), dict(metadata),
        data_parallel_mode, tuple(rank_local_shards), tuple(rank_runtime_states),
        {"fixed_axes": fixed, "resizable_axes": resizable, "rank_order_may_change": True,
         "model_shard_key": ["parameter_domain", "tp", "pp", "expert_ep"] if dcp
         else ["tp", "pp", "ep"],
         "optimizer_layout_requires_same_parameter_order": not dcp,
         "zero_bucket_boundaries_must_match": data_parallel_mode in ("zero1", "zero2", "zero3"),
         "shared_filesystem_required": bool(rank_local_shards) or dcp,
         "rng_exact_for_saved_coordinates": True,
         "new_replica_rng_policy": "keep_initialized_state_with_warning",
         "virtual_stages_per_rank": virtual_stages_per_rank},
        run_config, plan, virtual_stages_per_rank)


def validate_topology(manifest: CheckpointManifest, parallel) -> None:
    """TP/PP/CP sizes are fixed across resume; DP (and dense EP) may change."""
    if manifest.schema_version != SCHEMA_VERSION:
        raise ValueError(f"unsupported checkpoint schema {manifest.schema_version}; expected "
                         f"{SCHEMA_VERSION}")
    cur = parallel_sizes(parallel)
    for axis in ("tp", "pp", "cp"):
        saved = manifest.parallel_sizes.get(axis)
        if saved is not None and saved != cur[axis]:
            raise ValueError(f"phase-one checkpoint restore cannot change {axis.upper()} size "
                             f"({saved} -> {cur[axis]})")
    meta = list(manifest.tensor_metadata.values()) + [
        m for s in manifest.rank_local_shards for m in s.tensor_metadata.values()]
    saved_ep = manifest.parallel_sizes.get("ep")
    if saved_ep is not None and saved_ep != cur["ep"]:
        if any(m.parameter_domain is ParameterDomain.EXPERT for m in meta):
            raise ValueError("changing EP size for expert parameters requires an expert remap "
                             "planner")
        if manifest.data_parallel_mode == "zero3":
            raise ValueError(f"phase-one ZeRO-3 restore cannot change EP size: {saved_ep} -> "
                             f"{cur['ep']}")
