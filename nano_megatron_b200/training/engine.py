"""Assemble a training job from a :class:`TrainConfig` (the ``run`` path of the CLI).

Order of the reference's CLI (src/nano_megatron/cli/train.py:89-202): runtime ->
parallel context -> ParallelRNG -> ``torch.manual_seed(seed(DENSE_INIT))`` ->
context-parallel attention -> model builder (CPU init, fp32) -> data-parallel
strategy. The model is moved to the device and flattened into the strategy's
buffers in compute precision (bf16 on CUDA) with fp32 masters.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from nano_megatron_b200.context_parallel import build_context_parallel_attention
from nano_megatron_b200.data_parallel import build_data_parallel_strategy
from nano_megatron_b200.models.gpt import DenseGPTComponents, GPTModelBuilder
from nano_megatron_b200.parallel.context import ParallelContext
from nano_megatron_b200.parallel.domains import ParameterDomainRegistry
from nano_megatron_b200.parallel.rng import ParallelRNG, RNGStream


@dataclass
class TrainingComponents:
    runtime: object
    parallel: ParallelContext
    rng: ParallelRNG
    model: torch.nn.Module
    built: object
    data_parallel: object
    tp_workspace: object = None
    cp_heaps: list = None

    def close(self, trainer=None, *, keep_runtime: bool = False) -> None:
        """Ordered teardown: graphs, peer mappings, own buffer, subgroups and (unless
        ``keep_runtime``) the default group
        (:func:`nano_megatron_b200.distributed.shutdown.shutdown`)."""
        from nano_megatron_b200.distributed.shutdown import shutdown

        ws, self.tp_workspace = self.tp_workspace, None
        dp = self.data_parallel
        replica = getattr(dp, "replica", None)
        heaps = [(replica, dp.replica_group)] if replica is not None else []
        if replica is not None:
            dp.replica = None
        heaps += list(self.cp_heaps or [])
        self.cp_heaps = []
        from nano_megatron_b200.models.gpt.model import GPTModel

        for m in self.model.modules():
            core = getattr(m, "cp_attention", None) if isinstance(m, GPTModel) else None
            if core is not None and hasattr(core, "detach"):
                core.detach()
        shutdown(trainer=trainer, model=self.model, workspace=ws, parallel=self.parallel,
                 runtime=None if keep_runtime else self.runtime,
                 device=getattr(self.runtime, "device", None), heaps=heaps)


def build_model(config, parallel, rng, *, device):
    torch.manual_seed(rng.seed(RNGStream.DENSE_INIT))
    cp_attention = build_context_parallel_attention(config.context_parallel, parallel)
    components = DenseGPTComponents(cp_attention=cp_attention)
    builder = GPTModelBuilder(components, parameter_domains=ParameterDomainRegistry(),
                              activation_checkpoint_config=config.activation_checkpoint)
    if config.pipeline.virtual_stages_per_rank > 1:
        built = builder.build_pipeline(config.model, parallel, None,
                                       virtual_stages_per_rank=config.pipeline
                                       .virtual_stages_per_rank, rng=rng,
                                       cp_attention=cp_attention)
    else:
        built = builder.build_stage(config.model, parallel, None, rng=rng,
                                    cp_attention=cp_attention)
    model = built.model.to(device=device)
    return model, built


def build_training_components(config, runtime) -> TrainingComponents:
    from nano_megatron_b200.ops.deterministic import configure as configure_determinism

    configure_determinism(getattr(config.kernels, "deterministic", False))
    parallel = ParallelContext.create(runtime, config.parallel)
    rng = ParallelRNG.from_context(config.training.seed, parallel)
    model, built = build_model(config, parallel, rng, device=runtime.device)
    strategy = build_data_parallel_strategy(config.data_parallel, config.offload, parallel,
                                            built.parameter_domains)
    strategy.configure_precision(config.precision)
    from nano_megatron_b200.tensor_parallel.fused import attach_tp_workspace

    ws = attach_tp_workspace(model, config, parallel, torch.device(runtime.device))
    from nano_megatron_b200.context_parallel.fused import attach_cp_heap
    from nano_megatron_b200.models.gpt.model import GPTModel

    cores = {id(m.cp_attention): m.cp_attention for m in model.modules()
             if isinstance(m, GPTModel) and m.cp_attention is not None}
    cp_heaps = [attach_cp_heap(model, config, parallel, core, torch.device(runtime.device))
                for core in cores.values()]
    comps = TrainingComponents(runtime, parallel, rng, model, built, strategy, ws)
    comps.cp_heaps = [(h, parallel.cp) for h in cp_heaps if h is not None]
    return comps
