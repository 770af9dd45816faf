"""tcgen05 GEMM entry points.

The kernel computes ``C[m, n] = sum_k A(m, k) B(n, k)`` where either operand may
be stored K-major (``[rows, K]``) or MN-major (``[K, rows]``), so the forward,
input-gradient and weight-gradient products of a linear layer all run without
transposes. Fused epilogues: bf16 store (optional residual add and device
scalar scale), fp32 accumulate (weight gradients into fp32 main-grad buffers),
SwiGLU (gate/up projection), rotary embedding (QKV projection).

The reference computes these with ``nn.Linear`` / ``F.linear`` under autocast
(src/nano_megatron/nn/kernels/torch_backend.py:19-20,
src/nano_megatron/tensor_parallel/layers.py:214).
"""

from __future__ import annotations

import torch

from ._ext import lib, status_word

EPI_BF16, EPI_F32_ACC, EPI_SWIGLU, EPI_ROPE, EPI_CE_STATS = 0, 1, 2, 3, 5


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    epilogue: int = EPI_BF16,
    residual: torch.Tensor | None = None,
    alpha: float = 1.0,
    alpha_t: torch.Tensor | None = None,
    beta: float = 0.0,
    aux: torch.Tensor | None = None,
    swiglu_up_row: int = 0,
    positions: torch.Tensor | None = None,
    inv_freq: torch.Tensor | None = None,
    head_dim: int = 0,
    rope_cols: int = 0,
    pos_div: int = 1,
    block_n: int = 0,
    max_ctas: int = 0,
    rope_cs: torch.Tensor | None = None,
    ce_part: torch.Tensor | None = None,
) -> torch.Tensor:
    lib().gemm_tc(
        a, a_mn, b, b_mn, out, epilogue, residual, alpha_t, float(alpha), float(beta), aux,
        int(swiglu_up_row), positions, inv_freq, int(head_dim), int(rope_cols), int(pos_div),
        status_word(a.device), int(block_n), int(max_ctas), rope_cs, ce_part,
    )
    return out


def ce_parts_per_row(vocab: int) -> int:
    """(max, sum exp) parts per row the LM-head statistics epilogue writes: two per
    256-column tile."""
    return (vocab + 255) // 256 * 2


def lm_head_ce_stats(x: torch.Tensor, weight: torch.Tensor, *, out: torch.Tensor | None = None
                     ) -> tuple[torch.Tensor, torch.Tensor]:
    """``x @ weight.T`` (bf16 logits) and the per-row, per-tile (max, sum exp) of the
    rounded logits, ``[M, ce_parts_per_row(V), 2]`` fp32, from the same GEMM's epilogue."""
    m, v = x.shape[0], weight.shape[0]
    if out is None:
        out = torch.empty(m, v, device=x.device, dtype=torch.bfloat16)
    parts = torch.empty(m, ce_parts_per_row(v), 2, device=x.device, dtype=torch.float32)
    gemm(x, weight, out, epilogue=EPI_CE_STATS, ce_part=parts)
    return out, parts


_ROPE_TABLES: dict = {}


def rope_table(positions: torch.Tensor, inv_freq: torch.Tensor,
               dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``[len(positions), D/2, 2]`` table of (cos, sin)(position * inv_freq), computed in
    fp32 and stored as ``dtype``. The QKV GEMM's RoPE epilogue reads it as bf16 (the
    reference's rotary embedding also casts cos and sin to the compute dtype,
    src/nano_megatron/nn/rotary.py:36); the attention backward's inverse rotation reads it
    as fp32.

    Built once per positions tensor (the model caches those per sequence layout) and
    kept with a reference to it, so its address cannot be reused by another tensor
    while the entry lives."""
    key = (positions.data_ptr(), positions.numel(), inv_freq.data_ptr(), positions.device, dtype)
    hit = _ROPE_TABLES.get(key)
    if hit is not None:
        return hit[2]
    ang = positions.to(torch.float32)[:, None] * inv_freq.to(torch.float32)[None, :]
    table = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).to(dtype).contiguous()
    if len(_ROPE_TABLES) >= 64:
        _ROPE_TABLES.pop(next(iter(_ROPE_TABLES)))
    _ROPE_TABLES[key] = (positions, inv_freq, table)
    return table


def linear_fwd(x: torch.Tensor, weight: torch.Tensor, *, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T`` (+ residual) for 2-D bf16 ``x`` [M, K] and ``weight`` [N, K]."""
    if out is None:
        out = torch.empty(x.shape[0], weight.shape[0], device=x.device, dtype=torch.bfloat16)
    return gemm(x, weight, out, residual=residual)


def linear_dgrad(dy: torch.Tensor, weight: torch.Tensor, *, out: torch.Tensor | None = None,
                 alpha_t: torch.Tensor | None = None) -> torch.Tensor:
    """``dy @ weight`` for ``dy`` [M, N] and ``weight`` [N, K] (weight read MN-major)."""
    if out is None:
        out = torch.empty(dy.shape[0], weight.shape[1], device=dy.device, dtype=torch.bfloat16)
    return gemm(dy, weight, out, b_mn=True, alpha_t=alpha_t)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, main_grad: torch.Tensor, *,
                 accumulate: bool = True, alpha_t: torch.Tensor | None = None) -> torch.Tensor:
    """``main_grad (+)= dy.T @ x`` in fp32 (both operands read MN-major)."""
    return gemm(dy, x, main_grad, a_mn=True, b_mn=True, epilogue=EPI_F32_ACC,
                beta=1.0 if accumulate else 0.0, alpha_t=alpha_t)


def swiglu_fwd(x: torch.Tensor, w_gate_up: torch.Tensor, ffn: int, *,
               out: torch.Tensor | None = None, gate_up: torch.Tensor | None = None):
    """h = silu(x Wg^T) * (x Wu^T) with ``w_gate_up = [Wg; Wu]`` ([2F, H]).

    Returns ``(h [M, F], gate_up [M, 2F])``; ``gate_up`` is kept for backward.
    """
    m = x.shape[0]
    if out is None:
        out = torch.empty(m, ffn, device=x.device, dtype=torch.bfloat16)
    if gate_up is None:
        gate_up = torch.empty(m, 2 * ffn, device=x.device, dtype=torch.bfloat16)
    gemm(x, w_gate_up, out, epilogue=EPI_SWIGLU, aux=gate_up, swiglu_up_row=ffn)
    return out, gate_up


def qkv_rope_fwd(x: torch.Tensor, w_qkv: torch.Tensor, positions: torch.Tensor,
                 inv_freq: torch.Tensor, head_dim: int, rope_cols: int, *, pos_div: int = 1,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused QKV projection with rotary embedding on the first ``rope_cols`` columns."""
    if out is None:
        out = torch.empty(x.shape[0], w_qkv.shape[0], device=x.device, dtype=torch.bfloat16)
    return gemm(x, w_qkv, out, epilogue=EPI_ROPE, positions=positions, inv_freq=inv_freq,
                head_dim=head_dim, rope_cols=rope_cols, pos_div=pos_div,
                rope_cs=rope_table(positions, inv_freq, torch.bfloat16))
