"""Non-reentrant activation checkpointing with optional pinned-CPU offload.

``full`` mode recomputes whole layers (every ``block_interval``-th layer) and
``selective`` mode recomputes the attention and/or MLP block, as in the
reference (src/nano_megatron/nn/activation_checkpoint.py:24-131). Built on
``torch.utils.checkpoint(use_reentrant=False, preserve_rng_state=True)``;
the fused block functions recompute their forward kernels during backward.
"""

from __future__ import annotations

from contextlib import nullcontext

import torch
from torch.utils.checkpoint import checkpoint


class _OffloadHooks(torch.autograd.graph.saved_tensors_hooks):
    """Move saved tensors to pinned host memory and back on use."""

    def __init__(self, pin_memory: bool = True) -> None:
        def pack(t: torch.Tensor):
            if not t.is_cuda:
                return (None, t)
            host = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin_memory)
            host.copy_(t, non_blocking=True)
            return (t.device, host)

        def unpack(packed):
            device, t = packed
            return t if device is None else t.to(device, non_blocking=True)

        super().__init__(pack, unpack)


ActivationOffloadHooks = _OffloadHooks


def activation_checkpoint(function, *args, rng=None, offload_saved_tensors: bool = False):
    ctx = _OffloadHooks() if offload_saved_tensors else nullcontext()
    with ctx:
        return checkpoint(function, *args, use_reentrant=False, preserve_rng_state=True)


class ActivationCheckpoint:
    """Callable policy object: ``policy(fn, x)`` checkpoints when enabled."""

    def __init__(self, enabled: bool = True, offload_saved_tensors: bool = False) -> None:
        self.enabled = enabled
        self.offload_saved_tensors = offload_saved_tensors

    def __call__(self, function, *args):
        if not self.enabled:
            return function(*args)
        return activation_checkpoint(function, *args,
                                     offload_saved_tensors=self.offload_saved_tensors)
