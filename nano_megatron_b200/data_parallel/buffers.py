"""Flat parameter / gradient buffers and their reduction buckets.

All parameters of one model chunk live in ONE contiguous buffer (compute
dtype) and all gradients in ONE contiguous fp32 buffer with the same layout;
every ``Parameter.data`` and ``Parameter.main_grad`` is a view. Consequences:

* the weight-gradient GEMM epilogue accumulates straight into the reduction
  buffer (no per-step pack/unpack copy, unlike the reference's bucket
  pack/unpack, src/nano_megatron/data_parallel/buckets.py:166-207);
* fused QKV and gate|up weights are zero-copy views (adjacent parameters);
* the optimizer runs one fused kernel over the flat fp32 master buffer.

Buckets are contiguous ranges cut with the reference's rule (a new bucket
starts when the running *parameter-dtype* byte count would exceed
``bucket_bytes``; parameters grouped by domain/replica group,
src/nano_megatron/data_parallel/buckets.py:347-404) so ZeRO state metadata
(``parameter_names``, ``numel``, ``padded_numel``, ``shard_numel``) is
identical. Each bucket is padded to a multiple of the replica-group size so it
reduce-scatters into equal shards.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn

_ALIGN = 8  # elements; keeps every parameter view 16-byte aligned for TMA


@dataclass
class ParamSlice:
    name: str
    parameter: nn.Parameter
    start: int          # element offset inside the bucket
    end: int
    tensor_sharded: bool
    tied_source_rank: int | None
    sequence_parallel_grad: bool

    @property
    def numel(self) -> int:
        return self.end - self.start


class Bucket:
    """One contiguous range of the flat buffers, reduced as a unit."""

    def __init__(self, index: int, domain, group, slices: list[ParamSlice], offset: int,
                 numel: int) -> None:
        self.index = index
        self.domain = domain
        self.group = group
        self.slices = slices
        self.offset = offset          # element offset of the bucket in the flat buffers
        self.numel = numel            # unpadded logical size (sum of parameter sizes)
        self.world_size = getattr(group, "size", 1)
        self.rank = getattr(group, "rank", 0)
        self.shard_numel = math.ceil(self.numel / self.world_size)
        self.padded_numel = self.shard_numel * self.world_size
        self.shard_start = self.rank * self.shard_numel
        self.shard_end = min(self.shard_start + self.shard_numel, self.numel)
        self.param_data: torch.Tensor | None = None   # set by FlatBuffers
        self.grad_data: torch.Tensor | None = None

    @property
    def parameters(self) -> tuple[nn.Parameter, ...]:
        return tuple(s.parameter for s in self.slices)

    @property
    def defer_until_finalize(self) -> bool:
        return any(s.tied_source_rank is not None for s in self.slices)

    def shard_view(self, flat: torch.Tensor) -> torch.Tensor:
        """This rank's shard of a bucket-sized (padded) tensor."""
        return flat[self.rank * self.shard_numel:(self.rank + 1) * self.shard_numel]

    def metadata(self) -> dict:
        return {"index": self.index, "domain": getattr(self.domain, "value", str(self.domain)),
                "parameter_names": [s.name for s in self.slices], "numel": self.numel,
                "padded_numel": self.padded_numel, "shard_numel": self.shard_numel}


class FlatBuffers:
    """Owns the flat param/grad storage of a set of (unique) parameters."""

    def __init__(self, named_params: list[tuple[str, nn.Parameter]], *, domains, parallel,
                 bucket_bytes: int, param_dtype: torch.dtype, grad_dtype: torch.dtype,
                 device: torch.device, unit_key=None, allocate=None) -> None:
        """``unit_key(name)``: optional; a new bucket also starts whenever it changes, so
        buckets never straddle two sharding units (ZeRO-3 gathers one unit at a time).
        ``allocate(numel, param_dtype, grad_dtype) -> (param_flat, grad_flat)``: optional
        zeroed storage (e.g. peer-mapped memory); default fresh device tensors."""
        self.param_dtype = param_dtype
        self.grad_dtype = grad_dtype
        self.device = device
        groups: dict[tuple, list] = {}
        for name, p in named_params:
            placement = domains.get(p) if domains is not None else None
            domain = getattr(placement, "domain", "dense")
            key_name = getattr(placement, "replica_group", "dense_replica")
            group = _resolve_group(parallel, key_name)
            key = (str(domain), str(key_name))
            groups.setdefault(key, [domain, group, []])[2].append((name, p, placement))
        self.buckets: list[Bucket] = []
        total = 0
        layout = []  # (bucket, [(slice, numel)])
        esize = torch.empty((), dtype=param_dtype).element_size()
        for domain, group, items in groups.values():
            current, cur_bytes, cur_unit = [], 0, None
            for name, p, placement in items:
                nbytes = p.numel() * esize
                unit = unit_key(name) if unit_key is not None else None
                if current and (cur_bytes + nbytes > bucket_bytes or unit != cur_unit):
                    layout.append((domain, group, current))
                    current, cur_bytes = [], 0
                cur_unit = unit
                current.append((name, p, placement))
                cur_bytes += nbytes
            if current:
                layout.append((domain, group, current))
        for domain, group, items in layout:
            slices, cursor = [], 0
            for name, p, placement in items:
                start = cursor
                cursor = start + p.numel()
                slices.append(ParamSlice(
                    name, p, start, cursor, bool(getattr(placement, "tensor_sharded", False)),
                    getattr(p, "_nano_megatron_tied_source_rank", None),
                    bool(getattr(p, "sequence_parallel_grad", False))))
                cursor = -(-cursor // _ALIGN) * _ALIGN
            bucket = Bucket(len(self.buckets), domain, group, slices, total, cursor)
            # the bucket's storage is padded to equal shards (and alignment)
            padded = -(-bucket.padded_numel // _ALIGN) * _ALIGN
            bucket.storage_numel = padded
            self.buckets.append(bucket)
            total += padded
        self.numel = total
        if allocate is not None:
            self.param_flat, self.grad_flat = allocate(total, param_dtype, grad_dtype)
        else:
            self.param_flat = torch.zeros(total, dtype=param_dtype, device=device)
            self.grad_flat = torch.zeros(total, dtype=grad_dtype, device=device)
        for b in self.buckets:
            b.param_data = self.param_flat[b.offset:b.offset + b.storage_numel]
            b.grad_data = self.grad_flat[b.offset:b.offset + b.storage_numel]
            for s in b.slices:
                p = s.parameter
                src = p.data
                view = self.param_flat[b.offset + s.start:b.offset + s.end].view(src.shape)
                view.copy_(src.to(device=device, dtype=param_dtype))
                p.data = view
                p.main_grad = self.grad_flat[b.offset + s.start:b.offset + s.end].view(src.shape)

    def zero_grad(self) -> None:
        self.grad_flat.zero_()

    def slices(self):
        for b in self.buckets:
            for s in b.slices:
                yield b, s


def _resolve_group(parallel, key):
    if parallel is None:
        return None
    try:
        return parallel.group(key)
    except (KeyError, AttributeError):
        return None


def unique_named_parameters(model: nn.Module) -> list[tuple[str, nn.Parameter]]:
    seen, out = set(), []
    for name, p in model.named_parameters():
        if id(p) in seen or not p.requires_grad:
            continue
        seen.add(id(p))
        out.append((name, p))
    return out
