"""Vocabulary-parallel embedding: rows ``[V/TP, H]`` split over TP ranks.

Each rank looks up the ids of its vocabulary shard (zeros elsewhere); the
partial embeddings are summed over TP (all-reduce) or, under sequence
parallelism, reduce-scattered along the sequence. Init normal(0, init_std).
Reference: src/nano_megatron/tensor_parallel/embedding.py:22-75.
"""

from __future__ import annotations

import torch
from torch import nn

from nano_megatron_b200.ops import functional as F

from .comm import reduce_from_tensor_parallel_region, reduce_scatter_to_sequence_parallel_region
from .layers import tensor_parallel_group


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, vstart):
        ctx.save_for_backward(ids)
        ctx.vstart = vstart
        ctx.wshape = weight.shape
        ctx.wdtype = weight.dtype
        return F.embedding(ids, weight, vstart).view(*ids.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        acc = torch.zeros(ctx.wshape, dtype=torch.float32, device=dy.device)
        F.embedding_bwd(ids, dy.reshape(-1, ctx.wshape[1]).contiguous(), acc, ctx.vstart)
        return None, acc.to(ctx.wdtype), None


class VocabParallelEmbedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int, *, parallel, kernels=None,
                 sequence_parallel: bool = False, init_std: float = 0.02, device=None,
                 dtype=None) -> None:
        super().__init__()
        self.group = tensor_parallel_group(parallel)
        if num_embeddings % self.group.size:
            raise ValueError(f"num_embeddings ({num_embeddings}) must be divisible by TP size "
                             f"({self.group.size})")
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.sequence_parallel = sequence_parallel
        self.num_embeddings_per_partition = num_embeddings // self.group.size
        self.vocab_start_index = self.group.rank * self.num_embeddings_per_partition
        self.vocab_end_index = self.vocab_start_index + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim,
                                               device=device, dtype=dtype))
        nn.init.normal_(self.weight, mean=0.0, std=init_std)

    def forward(self, input_ids: torch.Tensor, *, sequence_dim: int = 1) -> torch.Tensor:
        out = _EmbeddingFn.apply(input_ids, self.weight, self.vocab_start_index)
        if self.sequence_parallel:
            return reduce_scatter_to_sequence_parallel_region(out, self.group,
                                                              sequence_dim=sequence_dim)
        return reduce_from_tensor_parallel_region(out, self.group)
