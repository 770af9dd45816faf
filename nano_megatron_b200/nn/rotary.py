"""Rotary position embedding (rotate-half convention).

``inv_freq = 1 / theta ** (arange(0, D, 2) / D)`` in fp32, exactly as the
reference (src/nano_megatron/nn/rotary.py:9-70). On the training path the
rotation is fused into the QKV GEMM epilogue (angle = position * inv_freq,
evaluated in fp32 per element) and its inverse into the attention backward;
this module provides the frequencies and the standalone apply functions.
"""

from __future__ import annotations

import torch
from torch import nn


def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    exponent = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    return (1.0 / (theta ** exponent)).to(device)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """q, k ``[B, H, S, D]``; cos/sin ``[S, D]`` (or broadcastable)."""
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, theta: float = 10_000.0) -> None:
        super().__init__()
        if head_dim % 2:
            raise ValueError("rotary head_dim must be even")
        self.head_dim = head_dim
        self.theta = float(theta)
        self.register_buffer("inv_freq", rope_inv_freq(head_dim, theta), persistent=False)

    def forward(self, position_ids: torch.Tensor, *, device=None, dtype=None):
        inv = self.inv_freq.to(device or position_ids.device)
        freqs = position_ids.to(inv.device).float()[..., None] * inv
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos(), emb.sin()
        if dtype is not None:
            cos, sin = cos.to(dtype), sin.to(dtype)
        return cos, sin
