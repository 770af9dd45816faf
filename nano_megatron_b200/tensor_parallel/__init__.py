"""Tensor and sequence parallelism: layers, collectives, vocab-parallel loss."""

from .comm import (
    all_gather_dim0,
    all_reduce,
    copy_to_tensor_parallel_region,
    gather_from_sequence_parallel_region,
    gather_from_tensor_parallel_region,
    reduce_from_tensor_parallel_region,
    reduce_scatter_dim0,
    reduce_scatter_to_sequence_parallel_region,
    register_sequence_parallel_gradient_hooks,
    scatter_to_sequence_parallel_region,
    scatter_to_tensor_parallel_region,
)
from .cross_entropy import VocabParallelCrossEntropy, vocab_parallel_ce_rows
from .embedding import VocabParallelEmbedding
from .layers import ColumnParallelLinear, RowParallelLinear, VocabParallelLinear, tensor_parallel_group

__all__ = [n for n in dir() if not n.startswith("_")]
