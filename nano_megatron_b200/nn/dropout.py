"""Topology-stable dropout.

Masks are drawn from a generator seeded by the ParallelRNG ACTIVATION stream
keyed by (layer, microbatch, global token offset of the local shard, op) -- the
keying of the reference, src/nano_megatron/nn/dropout.py:14-70 -- so a mask is
reproduced exactly by a rerun and by activation-checkpoint recomputation. The draw
itself (CPU generator or the Philox kernel on CUDA, over this framework's
sequence-major tensors) differs from the reference's, so with p > 0 the two
frameworks' losses agree statistically, not bit for bit. p = 0 (the default, and
every benchmark configuration) is a no-op and allocates nothing.
"""

from __future__ import annotations

from contextlib import contextmanager

import torch


class DropoutMask:
    """Callable forward (``y * mask / (1-p)``) with the matching ``backward``.

    On CUDA (bf16) the mask is a pure function of (seed, element index) computed by the
    Philox kernel (``_C.dropout_apply``) in both passes, so nothing is stored; on CPU a
    seeded torch generator draws the mask and it is kept for the backward pass."""

    def __init__(self, p: float, seed: int) -> None:
        self.p = float(p)
        self.seed = int(seed) & ((1 << 63) - 1)
        self.mask: torch.Tensor | None = None

    @staticmethod
    def _kernel_ok(t: torch.Tensor) -> bool:
        return t.is_cuda and t.dtype == torch.bfloat16

    def _kernel(self, t: torch.Tensor) -> torch.Tensor:
        from nano_megatron_b200.ops._ext import lib

        src = t.contiguous()
        out = torch.empty_like(src)
        lib().dropout_apply(src, out, self.p, self.seed)
        return out

    def _make(self, like: torch.Tensor) -> torch.Tensor:
        gen = torch.Generator(device=like.device)
        gen.manual_seed(self.seed)
        keep = torch.rand(like.shape, generator=gen, device=like.device) >= self.p
        return keep.to(like.dtype) / (1.0 - self.p)

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        if self._kernel_ok(y):
            return self._kernel(y)
        self.mask = self._make(y)
        return y * self.mask

    def backward(self, dy: torch.Tensor) -> torch.Tensor:
        if self._kernel_ok(dy):
            return self._kernel(dy)
        mask = self.mask if self.mask is not None else self._make(dy)
        return dy * mask


def make_dropout(p: float, *, training: bool, rng, layer: int, microbatch: int,
                 global_token_offset: int, op: str) -> DropoutMask | None:
    if not training or p <= 0.0:
        return None
    if rng is None:
        seed = torch.initial_seed() ^ (layer * 1000003 + microbatch * 9176 + global_token_offset)
    else:
        seed = rng.activation_seed(layer=layer, microbatch=microbatch,
                                   global_token_offset=global_token_offset, op=op)
    return DropoutMask(p, seed)


def parallel_dropout(x: torch.Tensor, p: float, *, training: bool, rng=None, layer: int = 0,
                     microbatch: int = 0, global_token_offset: int = 0,
                     op: str = "dropout") -> torch.Tensor:
    fn = make_dropout(p, training=training, rng=rng, layer=layer, microbatch=microbatch,
                      global_token_offset=global_token_offset, op=op)
    if fn is None:
        return x
    return _DropoutFn.apply(x, fn)


class _DropoutFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fn):
        ctx.fn = fn
        return fn(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.fn.backward(g), None


@contextmanager
def activation_rng_context(rng, tensor, *, layer: int, microbatch: int, global_token_offset: int,
                           op: str):
    """Seed torch's default generators from the ACTIVATION stream inside the block."""
    if rng is None:
        yield
        return
    seed = rng.activation_seed(layer=layer, microbatch=microbatch,
                               global_token_offset=global_token_offset, op=op)
    devices = [tensor.device.index] if tensor.is_cuda else []
    with torch.random.fork_rng(devices=devices):
        torch.manual_seed(seed)
        yield
