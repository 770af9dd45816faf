"""Layer partitioning over (virtual) pipeline stages.

Even split with the remainder on the earliest stages; stage 0 owns the
embedding, the last stage the final norm, LM head and loss. With ``v`` virtual
stages per rank, logical stage = chunk * PP + pp_rank. Reference:
src/nano_megatron/pipeline_parallel/partition.py:31-140.
"""

from __future__ import annotations

from dataclasses import dataclass


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
    pp_rank: int
    chunk: int
    logical_stage: int


def partition_layers(num_layers: int, pipeline_size: int) -> tuple[LayerPartition, ...]:
    if pipeline_size < 1:
        raise ValueError("pipeline_size must be positive")
    if num_layers < pipeline_size:
        raise ValueError("num_layers must be at least pipeline_size; empty stages are unsupported")
    base, extra = divmod(num_layers, pipeline_size)
    out, start = [], 0
    for stage in range(pipeline_size):
        end = start + base + (stage < extra)
        last = stage == pipeline_size - 1
        out.append(LayerPartition(stage, start, end, stage == 0, last, last))
        start = end
    return tuple(out)


def partition_for_rank(num_layers: int, pipeline_size: int, pipeline_rank: int) -> LayerPartition:
    if not 0 <= pipeline_rank < pipeline_size:
        raise ValueError("pipeline_rank is outside the pipeline")
    return partition_layers(num_layers, pipeline_size)[pipeline_rank]


@dataclass(frozen=True)
class VirtualPipelineLayout:
    num_layers: int
    pipeline_size: int
    virtual_stages_per_rank: int = 1

    def __post_init__(self) -> None:
        if self.pipeline_size < 1:
            raise ValueError("pipeline_size must be positive")
        if self.virtual_stages_per_rank < 1:
            raise ValueError("virtual_stages_per_rank must be positive")
        if self.num_layers < self.num_logical_stages:
            raise ValueError("num_layers must be at least pipeline_size * "
                             "virtual_stages_per_rank; empty chunks are unsupported")

    @property
    def num_logical_stages(self) -> int:
        return self.pipeline_size * self.virtual_stages_per_rank

    @property
    def partitions(self) -> tuple[LayerPartition, ...]:
        return partition_layers(self.num_layers, self.num_logical_stages)

    def address(self, pp_rank: int, chunk: int) -> PipelineStageAddress:
        if not 0 <= pp_rank < self.pipeline_size:
            raise ValueError("pp_rank is outside the pipeline")
        if not 0 <= chunk < self.virtual_stages_per_rank:
            raise ValueError("chunk is outside the virtual pipeline")
        return PipelineStageAddress(pp_rank, chunk, chunk * self.pipeline_size + pp_rank)

    def _from_logical(self, logical: int) -> PipelineStageAddress:
        chunk, pp_rank = divmod(logical, self.pipeline_size)
        return self.address(pp_rank, chunk)

    def partition(self, address: PipelineStageAddress) -> LayerPartition:
        if self.address(address.pp_rank, address.chunk) != address:
            raise ValueError(f"inconsistent pipeline stage address: {address}")
        return self.partitions[address.logical_stage]

    def local_partitions(self, pp_rank: int) -> tuple[LayerPartition, ...]:
        return tuple(self.partition(self.address(pp_rank, c))
                     for c in range(self.virtual_stages_per_rank))

    def previous(self, address: PipelineStageAddress) -> PipelineStageAddress | None:
        cur = self.address(address.pp_rank, address.chunk).logical_stage
        return None if cur == 0 else self._from_logical(cur - 1)

    def next(self, address: PipelineStageAddress) -> PipelineStageAddress | None:
        cur = self.address(address.pp_rank, address.chunk).logical_stage
        return None if cur == self.num_logical_stages - 1 else self._from_logical(cur + 1)

    def is_first(self, address: PipelineStageAddress) -> bool:
        return self.address(address.pp_rank, address.chunk).logical_stage == 0

    def is_last(self, address: PipelineStageAddress) -> bool:
        return (self.address(address.pp_rank, address.chunk).logical_stage
                == self.num_logical_stages - 1)
