"""Build the local GPT stage (or the v virtual chunks of an interleaved pipeline).

Same protocol as the reference builder (src/nano_megatron/models/gpt/builder.py:
48-327): partition layers for this PP rank, build GPTModel with ownership
flags, register parameter domains with TP shard dims (column 0, row 1, vocab
0), attach a tied-embedding synchronizer when PP > 1, and wrap in
GPTPipelineStage (``forward(hidden, batch)`` returns hidden states or the loss)
or GPTPipeline (v chunks).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

from torch import nn

from nano_megatron_b200.parallel.domains import ParameterDomain, ParameterDomainRegistry
from nano_megatron_b200.parallel.group_plan import GroupKey
from nano_megatron_b200.pipeline_parallel.partition import (
    LayerPartition,
    VirtualPipelineLayout,
    partition_for_rank,
)
from nano_megatron_b200.tensor_parallel.embedding import VocabParallelEmbedding
from nano_megatron_b200.tensor_parallel.layers import (
    ColumnParallelLinear,
    RowParallelLinear,
    VocabParallelLinear,
)

from .model import GPTModel
from .tied_embeddings import TiedEmbeddingSynchronizer


@dataclass(frozen=True)
class BuiltGPTStage:
    model: "GPTPipelineStage"
    partition: LayerPartition
    parameter_domains: ParameterDomainRegistry


@dataclass(frozen=True)
class BuiltGPTPipeline:
    model: "GPTPipeline"
    partitions: tuple[LayerPartition, ...]
    layout: VirtualPipelineLayout
    parameter_domains: ParameterDomainRegistry


_ABSENT = object()


def _batch_value(batch: Any, key: str, default: Any = _ABSENT) -> Any:
    if isinstance(batch, Mapping):
        if key in batch:
            return batch[key]
    elif batch is not None and hasattr(batch, key):
        return getattr(batch, key)
    if default is not _ABSENT:
        return default
    raise KeyError(f"pipeline batch is missing required field {key!r}")


class GPTPipelineStage(nn.Module):
    """Adapter from GPTModel to the pipeline schedule protocol."""

    def __init__(self, model: GPTModel, partition: LayerPartition, *,
                 tied_embeddings: TiedEmbeddingSynchronizer | None = None) -> None:
        super().__init__()
        self.model = model
        self.partition = partition
        self.tied_embeddings = tied_embeddings

    def _tied_weight(self):
        return self.model.embedding.weight if self.partition.owns_embedding \
            else self.model.lm_head.weight

    def synchronize_tied_embedding_weights(self) -> None:
        if self.tied_embeddings is not None:
            self.tied_embeddings.bind_weight(self._tied_weight())
            self.tied_embeddings.synchronize_weight()

    def synchronize_tied_embedding_gradients(self) -> None:
        if self.tied_embeddings is not None:
            self.tied_embeddings.bind_weight(self._tied_weight())
            self.tied_embeddings.synchronize_gradient()

    def forward(self, hidden_states, batch):
        input_ids = _batch_value(batch, "input_ids") if self.partition.owns_embedding else None
        labels = _batch_value(batch, "labels", None) if self.partition.owns_lm_head else None
        out = self.model(input_ids, labels=labels,
                         position_ids=_batch_value(batch, "position_ids", None),
                         hidden_states=hidden_states,
                         microbatch_index=int(_batch_value(batch, "_microbatch_index", 0)))
        if not self.partition.owns_lm_head:
            return out.hidden_states
        if out.loss is None:
            raise ValueError("the last GPT pipeline stage requires batch['labels']")
        return out.loss


class GPTPipeline(nn.Module):
    """All virtual chunks hosted by one physical pipeline rank."""

    def __init__(self, chunks, layout: VirtualPipelineLayout) -> None:
        super().__init__()
        if len(chunks) != layout.virtual_stages_per_rank:
            raise ValueError("the number of local chunks must match virtual_stages_per_rank")
        self.chunks = nn.ModuleList(chunks)
        self.layout = layout

    def chunk(self, chunk_id: int) -> GPTPipelineStage:
        if not 0 <= chunk_id < len(self.chunks):
            raise IndexError(f"virtual pipeline chunk {chunk_id} is out of range")
        return self.chunks[chunk_id]

    def sharding_units(self):
        return tuple(self.chunks)

    def synchronize_tied_embedding_weights(self) -> None:
        for c in self.chunks:
            c.synchronize_tied_embedding_weights()

    def synchronize_tied_embedding_gradients(self) -> None:
        for c in self.chunks:
            c.synchronize_tied_embedding_gradients()

    def forward(self, hidden_states, batch):
        raise RuntimeError("GPTPipeline contains multiple virtual chunks; call chunk(id) through "
                           "an interleaved pipeline schedule")


class GPTModelBuilder:
    def __init__(self, components=None, *, parameter_domains=None,
                 activation_checkpoint_config=None) -> None:
        self.components = components
        self.parameter_domains = parameter_domains
        self.activation_checkpoint_config = activation_checkpoint_config

    @staticmethod
    def register_parameter_domains(model: nn.Module, registry: ParameterDomainRegistry) -> None:
        dims: dict[int, int] = {}
        for m in model.modules():
            if isinstance(m, ColumnParallelLinear):
                dims[id(m.weight)] = 0
                if m.bias is not None:
                    dims[id(m.bias)] = 0
            elif isinstance(m, RowParallelLinear):
                dims[id(m.weight)] = 1
            elif isinstance(m, (VocabParallelEmbedding, VocabParallelLinear)):
                dims[id(m.weight)] = 0
                if getattr(m, "bias", None) is not None:
                    dims[id(m.bias)] = 0
        for name, p in model.named_parameters():
            d = dims.get(id(p))
            registry.register(p, ParameterDomain.DENSE, tensor_sharded=d is not None,
                              tensor_shard_dim=d, name=name)

    def _model(self, config, parallel, kernels, part: LayerPartition, rng, cp_attention):
        return GPTModel(config, parallel=parallel, kernels=kernels, rng=rng,
                        components=self.components,
                        cp_attention=cp_attention if cp_attention is not None else
                        getattr(self.components, "cp_attention", None),
                        activation_checkpoint_config=self.activation_checkpoint_config,
                        layer_start=part.start_layer, layer_end=part.end_layer,
                        owns_embedding=part.owns_embedding, owns_final_norm=part.owns_final_norm,
                        owns_lm_head=part.owns_lm_head)

    @staticmethod
    def _tied(config, parallel, model, part) -> TiedEmbeddingSynchronizer | None:
        if not getattr(config, "tie_embeddings", True) or parallel.pp.size == 1:
            return None
        if not (part.owns_embedding or part.owns_lm_head):
            return None
        if not parallel.has_group(GroupKey.EMBEDDING):
            raise RuntimeError("a tied GPT pipeline endpoint is missing its embedding group")
        weight = model.embedding.weight if part.owns_embedding else model.lm_head.weight
        return TiedEmbeddingSynchronizer(weight, parallel.group(GroupKey.EMBEDDING))

    def build_stage(self, config, parallel, kernels=None, *, rng=None, cp_attention=None
                    ) -> BuiltGPTStage:
        part = partition_for_rank(config.layers, parallel.pp.size, parallel.coordinate.pp)
        model = self._model(config, parallel, kernels, part, rng, cp_attention)
        registry = self.parameter_domains or ParameterDomainRegistry()
        stage = GPTPipelineStage(model, part,
                                 tied_embeddings=self._tied(config, parallel, model, part))
        self.register_parameter_domains(stage, registry)
        return BuiltGPTStage(stage, part, registry)

    def build_pipeline(self, config, parallel, kernels=None, *, virtual_stages_per_rank: int,
                       rng=None, cp_attention=None) -> BuiltGPTPipeline:
        layout = VirtualPipelineLayout(config.layers, parallel.pp.size, virtual_stages_per_rank)
        parts = layout.local_partitions(parallel.coordinate.pp)
        chunks = []
        for part in parts:
            model = self._model(config, parallel, kernels, part, rng, cp_attention)
            chunks.append(GPTPipelineStage(
                model, part, tied_embeddings=self._tied(config, parallel, model, part)))
        pipeline = GPTPipeline(chunks, layout)
        registry = self.parameter_domains or ParameterDomainRegistry()
        self.register_parameter_domains(pipeline, registry)
        return BuiltGPTPipeline(pipeline, parts, layout, registry)
