"""Logical view of a model's local state: tensors + per-tensor shard metadata.

For each state-dict entry: global shape (local shape times TP along the
tensor-parallel dim), global offset (local size times TP rank), sharded axes,
parameter domain and the replica coordinate (dp, ep, cp for dense parameters;
dp, cp for expert ones) — the reference's metadata
(src/nano_megatron/checkpoint/mapping.py:13-220). Tensors are detached CPU
clones: model parameters here are views of flat buffers, and saving a view
would otherwise serialise the whole buffer.
"""

from __future__ import annotations

from collections.abc import Iterator, Mapping
from dataclasses import dataclass, field
from typing import Any

import torch

from nano_megatron_b200.parallel.axes import ParallelAxis
from nano_megatron_b200.parallel.domains import ParameterDomain

from .manifest import ShardMetadata


def _replica_coordinate(parallel, domain: ParameterDomain) -> tuple[int, ...]:
    c = getattr(parallel, "coordinate", None)
    if c is None:
        return ()
    return (c.dp, c.ep, c.cp) if domain is ParameterDomain.DENSE else (c.dp, c.cp)


def infer_shard_metadata(key: str, tensor: torch.Tensor, *, domain: ParameterDomain, parallel,
                         tensor_sharded: bool = False, tensor_shard_dim: int | None = None
                         ) -> ShardMetadata:
    local = tuple(int(s) for s in tensor.shape)
    glob = list(local)
    off = [0] * len(local)
    axes: list[ParallelAxis] = []
    if tensor_shard_dim is not None:
        if tensor_shard_dim >= len(local):
            raise ValueError(f"tensor shard dim {tensor_shard_dim} is outside {key!r} with local "
                             f"shape {local}")
        tp = parallel.tp
        glob[tensor_shard_dim] = local[tensor_shard_dim] * tp.size
        off[tensor_shard_dim] = local[tensor_shard_dim] * tp.rank
        axes.append(ParallelAxis.TP)
    if tensor_sharded and ParallelAxis.TP not in axes:
        axes.append(ParallelAxis.TP)
    return ShardMetadata(key, tuple(glob), local, tuple(off), tuple(axes), domain,
                         _replica_coordinate(parallel, domain))


def iter_tensors(value: Any, prefix: str = "") -> Iterator[tuple[str, torch.Tensor]]:
    if isinstance(value, torch.Tensor):
        yield prefix, value
    elif isinstance(value, Mapping):
        for k, v in value.items():
            yield from iter_tensors(v, f"{prefix}.{k}" if prefix else str(k))
    elif isinstance(value, (list, tuple)):
        for i, v in enumerate(value):
            yield from iter_tensors(v, f"{prefix}.{i}" if prefix else str(i))


@dataclass
class ShardedState(Mapping):
    state: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)

    def __getitem__(self, k):
        return self.state[k]

    def __iter__(self):
        return iter(self.state)

    def __len__(self) -> int:
        return len(self.state)

    def validate(self) -> None:
        tensors = dict(iter_tensors(self.state))
        unknown = set(self.metadata) - set(tensors)
        if unknown:
            raise ValueError(f"metadata refers to missing tensor keys: {sorted(unknown)}")
        for k, m in self.metadata.items():
            if tuple(tensors[k].shape) != m.local_shape:
                raise ValueError(f"metadata local shape for {k!r} is {m.local_shape}, tensor "
                                 f"shape is {tuple(tensors[k].shape)}")

    @classmethod
    def from_model(cls, model: torch.nn.Module, *, parameter_domains, parallel,
                   dtype: torch.dtype | None = None) -> "ShardedState":
        named = dict(model.named_parameters(remove_duplicate=False))
        state, meta = {}, {}
        for key, value in model.state_dict().items():
            if not isinstance(value, torch.Tensor):
                state[key] = value
                continue
            t = value.detach()
            if dtype is not None and t.is_floating_point():
                t = t.to(dtype)
            state[key] = t.to("cpu", copy=True).clone()
            p = named.get(key)
            domain, sharded, dim = ParameterDomain.DENSE, False, None
            if p is not None and parameter_domains is not None:
                placement = parameter_domains.get(p)
                if placement is not None:
                    domain = placement.domain
                    sharded = placement.tensor_sharded
                    dim = placement.tensor_shard_dim
            meta[key] = infer_shard_metadata(key, state[key], domain=domain, parallel=parallel,
                                             tensor_sharded=sharded, tensor_shard_dim=dim)
        out = cls(state, meta)
        out.validate()
        return out
