"""Kernel backend: the reference's small kernel surface, served by this library's kernels.

The reference lets model code take its kernels from a backend object with three entry
points (src/nano_megatron/nn/kernels/interface.py:10-33): ``linear(in, out, **kw)`` and
``rms_norm(hidden, eps, **kw)`` build modules, ``local_attention(q, k, v, ...)`` runs
attention on ``[batch, heads, sequence, head_dim]`` tensors. The GPT of this framework
does not go through it (its layers are fused autograd blocks, ``models/gpt/blocks.py``),
but code written against that seam can use :func:`build_kernel_backend` here and get the
sm_100a kernels on CUDA tensors:

* ``linear``: an ``nn.Linear`` whose forward is the tcgen05 GEMM and whose backward runs
  the dgrad GEMM and the fp32-accumulating weight-gradient GEMM (bf16 tensors; feature
  sizes multiples of 8, as TMA needs 16-byte row pitches);
* ``rms_norm``: :class:`nano_megatron_b200.nn.norms.RMSNorm` (fused forward/backward);
* ``local_attention``: the tcgen05 flash-attention forward and backward, native GQA,
  causal with an optional query offset (``sequence_offset``, as for a context-parallel
  query block against keys from position 0); head_dim 64 or 128.

On CPU tensors the same calls run the PyTorch formulas the kernels are tested against.
``kernels.backend`` ``b200`` and ``torch`` both select this backend (``torch`` is the
reference's spelling and stays accepted).
"""

from __future__ import annotations

import math
from typing import Any, Protocol

import torch
from torch import Tensor, nn

from nano_megatron_b200.ops import functional as F

from .norms import RMSNorm


class KernelBackend(Protocol):
    name: str

    def linear(self, in_features: int, out_features: int, **kwargs: Any) -> nn.Module: ...

    def rms_norm(self, hidden_size: int, eps: float, **kwargs: Any) -> nn.Module: ...

    def local_attention(self, q: Tensor, k: Tensor, v: Tensor, **kwargs: Any) -> Tensor: ...


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        rows = x.reshape(-1, x.shape[-1]).contiguous()
        y = F.linear(rows, weight)
        if bias is not None:
            y = y + bias
        ctx.save_for_backward(rows, weight)
        ctx.has_bias = bias is not None
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        rows, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = F.linear_dgrad(dy2, weight).view(ctx.in_shape)
        if ctx.needs_input_grad[1]:
            acc = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
            F.linear_wgrad(dy2, rows, acc)
            dw = acc.to(weight.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0).to(dy.dtype)
        return dx, dw, db


class Linear(nn.Linear):
    """``nn.Linear`` (same parameters, initialisation and state dict) computed with the
    tcgen05 GEMMs on CUDA."""

    def forward(self, x: Tensor) -> Tensor:
        if x.is_cuda and (self.in_features % 8 or self.out_features % 8):
            raise ValueError(f"sm_100a linear needs feature sizes divisible by 8 (16-byte "
                             f"rows), got {self.in_features} -> {self.out_features}")
        return _LinearFn.apply(x, self.weight, self.bias)


class _AttentionFn(torch.autograd.Function):
    """Flash attention on [B, S, H, D] contiguous tensors (the kernels' layout)."""

    @staticmethod
    def forward(ctx, q, k, v, causal, q_offset, scale):
        o, lse = F.attention_fwd(q, k, v, causal=causal, q_offset=q_offset, softmax_scale=scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.args = (causal, q_offset, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        causal, q_offset, scale = ctx.args
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        F.attention_bwd(q, k, v, o, do.contiguous(), lse, dq, dk, dv, causal=causal,
                        q_offset=q_offset, softmax_scale=scale)
        return dq, dk, dv, None, None, None


class B200KernelBackend:
    """Linear, RMSNorm and local attention from this library's kernels."""

    name = "b200"

    def linear(self, in_features: int, out_features: int, **kwargs: Any) -> nn.Module:
        return Linear(in_features, out_features, **kwargs)

    def rms_norm(self, hidden_size: int, eps: float, **kwargs: Any) -> nn.Module:
        return RMSNorm(hidden_size, eps, **kwargs)

    def local_attention(self, q: Tensor, k: Tensor, v: Tensor, *, causal: bool = True,
                        sequence_offset: int = 0, dropout_p: float = 0.0,
                        scale: float | None = None, attention_mask: Tensor | None = None,
                        **_: Any) -> Tensor:
        """Attention of ``q`` [B, Hq, Sq, D] against ``k``/``v`` [B, Hkv, Sk, D]; query i
        sits at position ``sequence_offset + i`` and keys at 0.. for the causal mask."""
        if q.ndim != 4 or k.ndim != 4 or v.ndim != 4 or k.shape != v.shape:
            raise ValueError("local_attention takes q [B, Hq, Sq, D] and k, v [B, Hkv, Sk, D]")
        if q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1]:
            raise ValueError("q and k/v disagree on batch size or head_dim")
        if q.shape[1] % k.shape[1]:
            raise ValueError(f"{q.shape[1]} query heads cannot share {k.shape[1]} key/value "
                             "heads evenly")
        if attention_mask is not None:
            raise NotImplementedError("local_attention supports causal or full masks only")
        if dropout_p:
            raise NotImplementedError("attention-probability dropout is not implemented")
        s = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
        # the kernels take [B, S, H, D] with contiguous heads
        qb, kb, vb = (t.transpose(1, 2).contiguous() for t in (q, k, v))
        o = _AttentionFn.apply(qb, kb, vb, bool(causal), int(sequence_offset), float(s))
        return o.transpose(1, 2)


TorchKernelBackend = B200KernelBackend   # the reference's name for its default backend


def build_kernel_backend(config: Any, parallel: Any = None) -> KernelBackend:
    """The backend ``kernels.backend`` names (``b200``, or the reference's ``torch``)."""
    backend = getattr(config, "backend", config)
    value = str(getattr(backend, "value", backend))
    if value in ("b200", "torch"):
        return B200KernelBackend()
    raise ValueError(f"unknown kernel backend {value!r} (b200 or torch)")


__all__ = ["B200KernelBackend", "KernelBackend", "Linear", "TorchKernelBackend",
           "build_kernel_backend"]
