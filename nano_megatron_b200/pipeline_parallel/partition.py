"""Which transformer layers each (virtual) pipeline stage holds.

``L`` layers over ``S`` stages: every stage gets ``L // S`` layers and the first
``L % S`` stages one more, so stage ``s`` starts at ``s * (L // S) + min(s, L % S)``.
Stage 0 also holds the embedding, the last stage the final norm and the LM head (and the
loss). With ``v`` virtual stages per rank there are ``S = PP * v`` logical stages and
chunk ``c`` of pipeline rank ``r`` is logical stage ``c * PP + r``: a microbatch visits
rank 0..PP-1 with chunk 0, then again with chunk 1, and so on. The split and the
stage numbering are the reference's (src/nano_megatron/pipeline_parallel/partition.py),
since checkpoints name layers by stage.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class LayerPartition:
    stage: int
    start_layer: int
    end_layer: int
    owns_embedding: bool
    owns_final_norm: bool
    owns_lm_head: bool

    @property
    def num_layers(self) -> int:
        return self.end_layer - self.start_layer


@dataclass(frozen=True)
class PipelineStageAddress:
    """Logical stage ``logical_stage`` as chunk ``chunk`` of pipeline rank ``pp_rank``."""

    pp_rank: int
    chunk: int
    logical_stage: int


def _stage_start(stage: int, per: int, extra: int) -> int:
    return stage * per + min(stage, extra)


def partition_layers(num_layers: int, pipeline_size: int) -> tuple[LayerPartition, ...]:
    """The ``pipeline_size`` contiguous layer ranges, earliest stages the longest."""
    if pipeline_size < 1:
        raise ValueError(f"pipeline_size={pipeline_size}: need at least one stage")
    if num_layers < pipeline_size:
        raise ValueError(f"{num_layers} layers cannot fill {pipeline_size} stages (a stage "
                         "without layers is not supported)")
    per, extra = divmod(num_layers, pipeline_size)
    last = pipeline_size - 1
    return tuple(LayerPartition(s, _stage_start(s, per, extra), _stage_start(s + 1, per, extra),
                                owns_embedding=s == 0, owns_final_norm=s == last,
                                owns_lm_head=s == last)
                 for s in range(pipeline_size))


def partition_for_rank(num_layers: int, pipeline_size: int, pipeline_rank: int) -> LayerPartition:
    if pipeline_rank not in range(pipeline_size):
        raise ValueError(f"pipeline rank {pipeline_rank} is not in [0, {pipeline_size})")
    return partition_layers(num_layers, pipeline_size)[pipeline_rank]


@dataclass(frozen=True)
class VirtualPipelineLayout:
    """The chunk <-> logical stage table of an (interleaved) pipeline. A plain value:
    builders and schedules receive it, nothing keeps a global "virtual rank"."""

    num_layers: int
    pipeline_size: int
    virtual_stages_per_rank: int = 1
    _table: tuple = field(init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        pp, v = self.pipeline_size, self.virtual_stages_per_rank
        if pp < 1 or v < 1:
            raise ValueError(f"pipeline_size={pp} and virtual_stages_per_rank={v} must both "
                             "be at least 1")
        if self.num_layers < pp * v:
            raise ValueError(f"{self.num_layers} layers cannot fill {pp} x {v} pipeline "
                             "chunks (a chunk without layers is not supported)")
        table = tuple(PipelineStageAddress(s % pp, s // pp, s) for s in range(pp * v))
        object.__setattr__(self, "_table", table)

    @property
    def num_logical_stages(self) -> int:
        return self.pipeline_size * self.virtual_stages_per_rank

    @property
    def partitions(self) -> tuple[LayerPartition, ...]:
        return partition_layers(self.num_layers, self.num_logical_stages)

    def address(self, pp_rank: int, chunk: int) -> PipelineStageAddress:
        if pp_rank not in range(self.pipeline_size) or \
                chunk not in range(self.virtual_stages_per_rank):
            raise ValueError(f"(pp_rank={pp_rank}, chunk={chunk}) is outside a "
                             f"{self.pipeline_size} x {self.virtual_stages_per_rank} pipeline")
        return self._table[chunk * self.pipeline_size + pp_rank]

    def _checked(self, address: PipelineStageAddress) -> int:
        """Logical stage of ``address`` after checking its three fields agree."""
        if self.address(address.pp_rank, address.chunk) != address:
            raise ValueError(f"{address} does not match this layout's numbering")
        return address.logical_stage

    def partition(self, address: PipelineStageAddress) -> LayerPartition:
        return self.partitions[self._checked(address)]

    def local_partitions(self, pp_rank: int) -> tuple[LayerPartition, ...]:
        parts = self.partitions
        return tuple(parts[self.address(pp_rank, c).logical_stage]
                     for c in range(self.virtual_stages_per_rank))

    def previous(self, address: PipelineStageAddress) -> PipelineStageAddress | None:
        s = self._checked(address)
        return self._table[s - 1] if s > 0 else None

    def next(self, address: PipelineStageAddress) -> PipelineStageAddress | None:
        s = self._checked(address)
        return self._table[s + 1] if s + 1 < len(self._table) else None

    def is_first(self, address: PipelineStageAddress) -> bool:
        return self._checked(address) == 0

    def is_last(self, address: PipelineStageAddress) -> bool:
        return self._checked(address) == len(self._table) - 1
