"""Fused data-parallel step over NVLink peer memory: gradient reduction + sharded AdamW +
bf16 parameter all-gather (the kernels are in ``csrc/dp_comm.cu``).

Replaces, for DDP and ZeRO-1/2 on one node, the reference's bucket all-reduce
(src/nano_megatron/data_parallel/buckets.py:210-303) and the ZeRO reduce-scatter ->
sharded AdamW -> parameter all-gather sequence
(src/nano_megatron/data_parallel/_zero.py:166-199). Each rank's flat gradient and
parameter buffers live in one :class:`SymmetricHeap` region each, mapped by every
replica; a step is

    signal(GRAD) -> per bucket: replica_reduce (peer loads, in-place sum of this rank's
    shard, partial squared norms) -> device clip coefficient -> per bucket:
    replica_adamw_gather (AdamW on the shard, bf16 stores into every replica's
    parameter buffer) -> signal(PARAM) -> replica_wait(PARAM).

Every rank owns the same contiguous shard of each bucket as under ZeRO (the reference's
``ceil(numel / world)`` cut), so under DDP the fp32 master and moments outside this
rank's shards are not updated; :meth:`gather_state` refreshes them from their owners
before a checkpoint is written.
"""

from __future__ import annotations

import os

import torch

CH_GRAD, CH_PARAM = 0, 1
_FLAG_BYTES = 4096


def fused_replica_supported(strategy, device: torch.device) -> tuple[bool, str]:
    """Whether ``strategy`` can run the fused replica path; returns (ok, reason)."""
    g = strategy.replica_group
    if device.type != "cuda":
        return False, "not on CUDA"
    if not getattr(strategy, "fused_replica_enabled", False):
        return False, "kernels.fused_dp_comm is off"
    if g is None or g.size <= 1:
        return False, "no replica group"
    if g.size > 8:
        return False, "more than 8 replicas"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("LOCAL_WORLD_SIZE", world)) != world:
        return False, "replicas span several nodes"
    if strategy.mode not in ("ddp", "zero1", "zero2"):
        return False, f"mode {strategy.mode}"
    if strategy.offload_policy.optimizer_state:
        return False, "optimizer state is offloaded"
    dt = strategy.grad_reduce_dtype
    if dt is not None and dt != torch.float32:
        return False, "precision.grad_reduce below fp32 (kept on NCCL in that dtype)"
    return True, ""


class ReplicaComm:
    def __init__(self, heap, group) -> None:
        self.heap = heap
        self.group = group
        self.n = heap.size
        self.rank = heap.rank
        self.segments: dict[int, torch.Tensor] = {}
        self.partials: dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------ construction
    @staticmethod
    def regions(numel: int, param_dtype: torch.dtype, grad_dtype: torch.dtype) -> dict:
        pe = torch.empty((), dtype=param_dtype).element_size()
        ge = torch.empty((), dtype=grad_dtype).element_size()
        return {"flags": _FLAG_BYTES, "grad": numel * ge, "param": numel * pe}

    @classmethod
    def create(cls, group, numel: int, param_dtype, grad_dtype, device) -> "ReplicaComm":
        from nano_megatron_b200.distributed.symmetric import SymmetricHeap

        heap = SymmetricHeap.create(group, cls.regions(numel, param_dtype, grad_dtype), device)
        return cls(heap, group)

    def flat_tensors(self, numel: int, param_dtype, grad_dtype):
        p = self.heap.local("param", param_dtype)[:numel]
        g = self.heap.local("grad", grad_dtype)[:numel]
        return p, g

    def prepare(self, buffers, counts) -> None:
        """Per bucket: this rank's norm-counted ranges (relative to its shard) and the
        partials buffer. ``counts(slice) -> bool`` is the norm counting rule."""
        from nano_megatron_b200.ops._ext import lib

        dev = buffers.device
        index = dev.index if dev.index is not None else torch.cuda.current_device()
        for b in buffers.buckets:
            lo = b.rank * b.shard_numel
            hi = lo + b.shard_numel
            segs: list[list[int]] = []
            for s in b.slices:
                a, e = max(s.start, lo), min(s.end, hi)
                if a >= e or not counts(s):
                    continue
                if segs and segs[-1][1] >= a:
                    segs[-1][1] = max(segs[-1][1], e)
                else:
                    segs.append([a, e])
            flat = [x - lo for seg in segs for x in seg]
            self.segments[b.index] = torch.tensor(flat, dtype=torch.int64, device=dev)
            blocks = int(lib().replica_reduce_blocks(b.shard_numel, index))
            self.partials[b.index] = torch.zeros(blocks, dtype=torch.float32, device=dev)

    # ------------------------------------------------------------------ step phases
    def _grad_ptrs(self) -> list[int]:
        return [self.heap.ptr(r, "grad") for r in range(self.n)]

    def _param_ptrs(self) -> list[int]:
        return [self.heap.ptr(r, "param") for r in range(self.n)]

    def signal(self, channel: int) -> None:
        from nano_megatron_b200.ops._ext import lib

        lib().peer_signal(self.heap.signal_targets(channel), self.heap.epoch_ptr(channel))

    def reduce(self, b, elem_offset_of) -> torch.Tensor:
        """Sum this rank's shard of bucket ``b`` over the replicas (in place); returns the
        bucket's partial squared norms (device)."""
        from nano_megatron_b200.ops._ext import lib

        off = elem_offset_of(b) + b.rank * b.shard_numel
        lib().replica_reduce(self._grad_ptrs(), self.rank, off, b.shard_numel,
                             self.segments[b.index], self.partials[b.index],
                             self.heap.flag_slots(self.rank, CH_GRAD),
                             self.heap.epoch_ptr(CH_GRAD), self.heap.status)
        return self.partials[b.index]

    def adamw_gather(self, b, elem_offset_of, master, exp_avg, exp_avg_sq, *, lr, betas, eps,
                     wd, step, grad_scale, lr_t) -> None:
        from nano_megatron_b200.ops._ext import lib

        off = elem_offset_of(b) + b.rank * b.shard_numel
        lib().replica_adamw_gather(self._grad_ptrs(), self._param_ptrs(), self.rank, off,
                                   b.shard_numel, master, exp_avg, exp_avg_sq, lr, betas[0],
                                   betas[1], eps, wd, step, grad_scale, lr_t)

    def wait(self, channel: int) -> None:
        from nano_megatron_b200.ops._ext import lib

        lib().replica_wait(self.heap.flag_slots(self.rank, channel), self.n,
                           self.heap.epoch_ptr(channel), self.heap.status)

    # ------------------------------------------------------------------ teardown
    def close(self) -> None:
        self.heap.close()

    def release(self) -> None:
        self.heap.release()
