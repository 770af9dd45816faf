"""Component factory hook (dense components; an MoE MLP could replace ``build_mlp``).

Reference: src/nano_megatron/models/gpt/factory.py:19-113.
"""

from __future__ import annotations

from typing import Protocol

from nano_megatron_b200.nn.norms import RMSNorm


class GPTComponentFactory(Protocol):
    def build_norm(self, config): ...

    def build_mlp(self, config, layer_index: int, *, parallel, sequence_parallel: bool): ...


class DenseGPTComponents:
    def __init__(self, *, cp_attention=None, sequence_parallel: bool | None = None) -> None:
        self.cp_attention = cp_attention
        self.sequence_parallel = sequence_parallel

    def build_norm(self, config, **_):
        return RMSNorm(config.hidden_size, float(getattr(config, "norm_epsilon", 1e-5)))

    def build_mlp(self, config, layer_index: int, *, parallel, sequence_parallel: bool):
        from .model import GPTMLP

        return GPTMLP(config, layer_index, parallel=parallel, sequence_parallel=sequence_parallel)
