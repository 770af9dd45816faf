"""RMSNorm module (parameter holder + functional forward).

Semantics of the reference (src/nano_megatron/nn/norms.py:13-41): normalise in
fp32, cast back to the input dtype, scale by the weight in that dtype; weight
initialised to ones. Inside GPT layers the norm runs fused in the layer
functions; this module's ``forward`` is the standalone autograd form.
"""

from __future__ import annotations

import torch
from torch import nn

from nano_megatron_b200.ops import functional as F


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y, rstd = F.rmsnorm(x2, weight, eps)
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        wgrad = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        dx = F.rmsnorm_bwd(x2, weight, dy.reshape(x2.shape).contiguous(), rstd, wgrad)
        return dx.view(ctx.shape), wgrad.to(weight.dtype), None


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-5, *, device=None, dtype=None) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = float(eps)
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _RMSNormFn.apply(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.hidden_size}, eps={self.eps}"
