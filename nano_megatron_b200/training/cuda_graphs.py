"""CUDA-graph capture of one microbatch's forward + backward (launch-bound loop -> one replay).

A training step of the GPT stage launches a few hundred kernels per microbatch
from Python; at B200 speeds the host cannot issue them as fast as the GPU
retires them. The microbatch is therefore captured once (per input shape) into
a CUDA graph -- forward, loss scaling, autograd backward, weight-gradient
accumulation into the fp32 ``main_grad`` buffers -- and replayed for every
microbatch after copying its token ids and labels into the graph's static
input buffers. Everything the graph touches has a fixed address: parameters
and gradients are views of the data-parallel flat buffers, activations come
from the graph's private memory pool, and no kernel on this path synchronises
with the host.

Capture protocol: one eager warm-up microbatch on a side stream (lazy kernel
attributes, cached positions, workspaces), then capture, then the gradient
buffers are zeroed again because warm-up accumulated into them. Used by the
no-pipeline schedule when ``kernels.cuda_graphs`` is on and the data-parallel
strategy does no per-microbatch communication. Tensor-parallel layers are
captured too: their NCCL collectives are graph-capturable, and the fused NVLink
collectives keep their flag epochs in device memory, so every replay advances
them like an eager call would.
"""

from __future__ import annotations

import torch


def _static_like(t: torch.Tensor, device) -> torch.Tensor:
    return torch.empty(t.shape, dtype=t.dtype, device=device)


class GraphedMicrobatch:
    def __init__(self, stage, data_parallel, template: dict, num_microbatches: int,
                 device: torch.device) -> None:
        self.stage = stage
        self.dp = data_parallel
        self.m = num_microbatches
        self.device = device
        self.keys = [k for k, v in template.items() if isinstance(v, torch.Tensor)]
        self.static = {k: _static_like(template[k], device) for k in self.keys}
        for k, v in template.items():
            if not isinstance(v, torch.Tensor):
                self.static[k] = v
        self.graph: torch.cuda.CUDAGraph | None = None
        self.out: torch.Tensor | None = None

    def _load(self, mb: dict) -> None:
        for k in self.keys:
            self.static[k].copy_(mb[k], non_blocking=True)

    def _step(self) -> torch.Tensor:
        # A captured microbatch is never the gradient-synchronising one: outside these
        # contexts a strategy's backward hooks (the overlap reducer) would launch
        # reductions that the graph would then replay on every microbatch.
        with self.dp.forward_microbatch_context(synchronize_gradients=False):
            out = self.stage(None, self.static)
        with self.dp.microbatch_context(is_last_microbatch=False):
            (out / self.m).backward()
        return out.detach()

    def capture(self, mb: dict) -> None:
        self._load(mb)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._step()                     # warm-up (accumulates into main_grad)
        torch.cuda.current_stream(self.device).wait_stream(side)
        from nano_megatron_b200.ops._ext import lib

        g = torch.cuda.CUDAGraph()
        before = lib().launch_count()
        with torch.cuda.graph(g):
            self.out = self._step()
        # Library kernels recorded into the graph; every replay launches them again.
        self.kernels = lib().launch_count() - before
        self.graph = g
        self.dp.zero_grad()                  # drop the warm-up's gradient contribution

    def release(self) -> None:
        """Free the graph and its static buffers (the graph's memory pool goes with it)."""
        self.graph = None
        self.out = None
        self.static = {}

    def run(self, mb: dict) -> torch.Tensor:
        from nano_megatron_b200.ops._ext import lib

        self._load(mb)
        self.graph.replay()
        lib().record_graph_launches(self.kernels)
        return self.out


def graph_key(mb: dict) -> tuple:
    return tuple(sorted((k, tuple(v.shape), v.dtype) for k, v in mb.items()
                        if isinstance(v, torch.Tensor)))


def graphs_supported(config, model, data_parallel, device: torch.device) -> bool:
    if device.type != "cuda" or not bool(getattr(config.kernels, "cuda_graphs", True)):
        return False
    if not getattr(data_parallel, "graph_safe_microbatches", False):
        return False
    if float(getattr(config.model, "dropout", 0.0)) > 0:
        return False
    if str(getattr(config.activation_checkpoint, "mode", "none")) != "none":
        return False
    return True
