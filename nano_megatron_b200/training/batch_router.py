"""Batch routing: the BATCH_REPLICA source rank feeds its TP/PP/CP peers.

The reference pickles each batch and broadcasts it as a Python object every
step (src/nano_megatron/training/batch_router.py:30-121). Here the source
moves the token tensors to the device once and broadcasts them as tensors over
the batch-replica communicator (NCCL over NVLink), then every rank slices its
context-parallel part (contiguous or zigzag). The key/shape/dtype header is sent
once: batches keep one layout for the life of the router (the source raises
before sending a batch of another layout).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from nano_megatron_b200.context_parallel.utils import shard_sequence
from nano_megatron_b200.parallel.group_plan import GroupKey

SEQUENCE_KEYS = ("input_ids", "labels", "position_ids", "loss_mask")


def shard_batch_for_context_parallel(batch: dict, rank: int, size: int, *,
                                     load_balance: bool = False) -> dict:
    if size == 1:
        return batch
    out = dict(batch)
    for k in SEQUENCE_KEYS:
        v = out.get(k)
        if isinstance(v, torch.Tensor) and v.ndim >= 2:
            out[k] = shard_sequence(v, rank, size, load_balance=load_balance, dim=1).contiguous()
    return out


class BatchRouter:
    def __init__(self, parallel, *, load_balance: bool = False) -> None:
        self.parallel = parallel
        self.load_balance = load_balance
        try:
            self.group = parallel.group(GroupKey.BATCH_REPLICA)
        except (KeyError, AttributeError):
            self.group = None
        self._shape_cache: dict = {}

    @property
    def is_source(self) -> bool:
        return self.group is None or self.group.rank == 0

    def _broadcast(self, batch):
        g = self.group
        if g is None or g.size == 1:
            return batch
        src = g.ranks[0]
        dev = torch.device("cuda", torch.cuda.current_device()) if g.backend == "nccl" \
            else torch.device("cpu")
        if self.is_source:
            keys = sorted(k for k, v in batch.items() if isinstance(v, torch.Tensor))
            header = [(k, tuple(batch[k].shape), str(batch[k].dtype)) for k in keys]
        else:
            header = None
        cached = self._shape_cache.get("header")
        if cached is None:
            # The key / shape / dtype header crosses once; later steps send tensors only,
            # so the peers never wait on the host for the source.
            box = [header]
            dist.broadcast_object_list(box, src=src, group=g.process_group)
            self._shape_cache["header"] = cached = box[0]
        elif self.is_source and header != cached:
            # The peers post receives of the cached shapes; sending others would mismatch.
            raise ValueError(f"batch layout changed after the first step: {header} != "
                             f"{cached}; the peers of a batch-replica group need batches of "
                             "one fixed shape")
        header = cached
        out = {}
        for k, shape, dt in header:
            dtype = getattr(torch, dt.replace("torch.", ""))
            # contiguous: loaders hand out views (input_ids / labels slice one [B, S+1]
            # buffer) and a collective sends the tensor's storage as laid out
            t = batch[k].to(dev).contiguous() if self.is_source else \
                torch.empty(shape, dtype=dtype, device=dev)
            dist.broadcast(t, src=src, group=g.process_group)
            out[k] = t
        return out

    def route(self, batch):
        batch = self._broadcast(batch)
        cp = self.parallel.cp
        return shard_batch_for_context_parallel(batch, cp.rank, cp.size,
                                                load_balance=self.load_balance)
