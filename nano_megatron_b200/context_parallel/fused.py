"""Attach the NVLink peer-memory transport of the ring context-parallel attention.

Created once per CP group (a collective over it) when training on CUDA with the ring
backend, ``kernels.fused_cp_comm`` on, at most 8 CP ranks on one node and no pipeline
parallelism (a layer's K/V slot is reused by the next microbatch, which with several
microbatches in flight per stage would need one slot per microbatch). Heap regions per
rank: flags; one K/V slot per local layer ([S_local, B, 2 * Hkv_local * D] bf16, kept
from the layer's forward to its backward); fp32 dK/dV return slots, 2 parities x CP
source ranks.
"""

from __future__ import annotations

import os

import torch


def wants_fused_cp(config, parallel, cp_attention, device) -> bool:
    from .attention import PeerRingContextParallelAttention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    return (isinstance(cp_attention, PeerRingContextParallelAttention) and
            device.type == "cuda" and 1 < parallel.cp.size <= 8 and parallel.pp.size == 1 and
            bool(getattr(config.kernels, "fused_cp_comm", True)) and
            int(os.environ.get("LOCAL_WORLD_SIZE", world)) == world)


def attach_cp_heap(model: torch.nn.Module, config, parallel, cp_attention, device):
    """Create the heap (collective over CP) and attach it to ``cp_attention``; returns
    the heap, or None when the layout keeps the NCCL ring."""
    if not wants_fused_cp(config, parallel, cp_attention, device):
        return None
    from nano_megatron_b200.distributed.symmetric import SymmetricHeap
    from nano_megatron_b200.models.gpt.model import GPTLayer

    m = config.model
    tp = parallel.tp.size
    s_local = int(m.seq_length) // parallel.cp.size
    head_dim = int(m.hidden_size) // int(m.heads)
    kv_heads = int(m.num_kv_heads) // tp
    kv_numel = s_local * int(config.training.micro_batch_size) * 2 * kv_heads * head_dim
    layers = sorted(mod.layer_index for mod in model.modules() if isinstance(mod, GPTLayer))
    slots = {layer: i for i, layer in enumerate(layers)}
    n = parallel.cp.size
    heap = SymmetricHeap.create(parallel.cp, {"flags": 4096, "kv": len(layers) * kv_numel * 2,
                                              "dkv": 2 * n * kv_numel * 4}, device)
    cp_attention.attach(heap, slots, kv_numel, device)
    return heap
