"""Gradient accumulation without pipeline parallelism (PP = 1)."""

from __future__ import annotations

import torch

from nano_megatron_b200.utils.profiling import nvtx_range

from .base import LossAccumulator, batch_labels, extract_loss


class NoPipelineSchedule:
    """Gradient accumulation over microbatches; with ``use_graphs`` each training microbatch
    is one CUDA-graph replay (:mod:`nano_megatron_b200.training.cuda_graphs`)."""

    def __init__(self, stage, data_parallel, *, use_graphs: bool = False) -> None:
        self.stage = stage
        self.data_parallel = data_parallel
        self.use_graphs = use_graphs
        self._graphs: dict = {}

    def _graphed(self, microbatches, acc: LossAccumulator) -> None:
        from nano_megatron_b200.training.cuda_graphs import GraphedMicrobatch, graph_key

        m = len(microbatches)
        keys = [(graph_key(mb), m) for mb in microbatches]
        if self.data_parallel.eager_last_microbatch():
            keys[-1] = None
        # Capture every missing shape before running any microbatch: a capture's warm-up
        # zeroes the gradient buffers, which must not erase this step's accumulation.
        for key, mb in zip(keys, microbatches):
            if key is not None and key not in self._graphs:
                device = next(self.stage.parameters()).device
                g = GraphedMicrobatch(self.stage, self.data_parallel, mb, m, device)
                g.capture(mb)
                self._graphs[key] = g
        eager_last = self.data_parallel.eager_last_microbatch()
        for i, (key, mb) in enumerate(zip(keys, microbatches)):
            if eager_last and i == m - 1:
                # the overlap reducer communicates from this backward: not graph-replayable
                dp = self.data_parallel
                with dp.forward_microbatch_context(synchronize_gradients=True):
                    loss = extract_loss(self.stage(None, mb), mb, m, acc)
                with dp.microbatch_context(is_last_microbatch=True):
                    dp.backward(loss)
                continue
            with nvtx_range(f"graph mb {i}"):
                acc.add(self._graphs[key].run(mb).clone(), batch_labels(mb))

    def release_graphs(self) -> None:
        graphs, self._graphs = self._graphs, {}
        for g in graphs.values():
            g.release()

    def forward_backward(self, microbatches, *, forward_only: bool = False
                         ) -> LossAccumulator:
        acc = LossAccumulator()
        m = len(microbatches)
        dp = self.data_parallel
        if self.use_graphs and not forward_only:
            self._graphed(microbatches, acc)
            return acc
        for i, mb in enumerate(microbatches):
            last = i == m - 1
            if forward_only:
                with torch.no_grad(), nvtx_range(f"eval mb {i}"):
                    extract_loss(self.stage(None, mb), mb, m, acc)
                continue
            with dp.forward_microbatch_context(synchronize_gradients=last), \
                    nvtx_range(f"fwd mb {i}"):
                loss = extract_loss(self.stage(None, mb), mb, m, acc)
            with dp.microbatch_context(is_last_microbatch=last), nvtx_range(f"bwd mb {i}"):
                dp.backward(loss)
        return acc
