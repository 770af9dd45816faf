"""Context parallelism: the sequence is split over CP ranks.

Two attention cores plug into the fused attention block
(:class:`nano_megatron_b200.models.gpt.blocks.LocalAttentionCore` interface):

* ``all_gather`` — K/V of every CP rank are gathered once, each rank runs the
  causal flash kernels for its query rows against the full K/V; the K/V
  gradients are reduce-scattered back (reference: src/nano_megatron/
  context_parallel/all_gather.py:38-113, which materialises a boolean mask and
  calls SDPA);
* ``ring`` — K/V blocks travel around the CP ring; each step runs the flash
  kernel on the resident block and merges partial outputs by log-sum-exp, and
  fully-masked blocks are skipped (reference: context_parallel/ring.py:104-322,
  which materialises fp32 score blocks and computes masked blocks).

Chunking: contiguous (rank r holds positions [r*S/CP, (r+1)*S/CP), the
reference's layout) or, with ``context_parallel.load_balance``, zigzag (rank r
holds chunks r and 2*CP-1-r of 2*CP equal chunks) so causal work is balanced.
"""

from __future__ import annotations

from .attention import (AllGatherContextParallelAttention, ContextParallelAttention,
                        PeerAllGatherContextParallelAttention, PeerRingContextParallelAttention,
                        RingContextParallelAttention)
from .utils import local_positions, shard_sequence, unshard_sequence


def build_context_parallel_attention(config, parallel):
    if parallel.cp.size == 1:
        return None
    backend = str(getattr(config.backend, "value", config.backend))
    balance = bool(getattr(config, "load_balance", False))
    if backend == "all_gather":
        # the peer-memory gather / reduce-scatter is attached later (attach_cp_heap) when the
        # layout allows it; until then (and on CPU) this core runs the NCCL all-gather
        return PeerAllGatherContextParallelAttention(parallel.cp, load_balance=balance)
    if backend == "ring":
        # the peer-memory transport is attached later (attach_cp_heap) when the layout
        # allows it; until then (and on CPU) this core runs the NCCL ring
        return PeerRingContextParallelAttention(parallel.cp, load_balance=balance)
    raise ValueError(f"unknown context-parallel backend {backend!r}")


__all__ = ["AllGatherContextParallelAttention", "ContextParallelAttention",
           "PeerAllGatherContextParallelAttention",
           "PeerRingContextParallelAttention",
           "RingContextParallelAttention",
           "build_context_parallel_attention", "local_positions", "shard_sequence",
           "unshard_sequence"]
