"""Leaf operations used by the model, one function per fused kernel.

Each function runs this library's sm_100a kernel when its inputs live on a CUDA
device, and the equivalent PyTorch formula when they live on the CPU. The CPU
formulas exist so that the multi-process gloo tests, CPU smoke runs and
parity checks against the reference can run without a GPU; they are not a
selectable backend (on a CUDA tensor the kernel is mandatory and a missing
library raises).

Shapes: activations are 2-D ``[tokens, features]`` row-major; attention takes
``[B, S, H, D]`` strided views (see :mod:`.attention`).
"""

from __future__ import annotations

import math

import torch

from . import gemm as _g
from ._ext import lib


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


# ------------------------------------------------------------------ GEMMs
def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ residual)``."""
    if _cuda(x):
        return _g.linear_fwd(x, w, residual=residual, out=out)
    y = x @ w.t()
    if residual is not None:
        y = y + residual
    if out is not None:
        out.copy_(y)
        return out
    return y


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, alpha_t: torch.Tensor | None = None
                 ) -> torch.Tensor:
    """``dy @ w`` (optionally scaled by the device scalar ``alpha_t``)."""
    if _cuda(dy):
        return _g.linear_dgrad(dy, w, alpha_t=alpha_t)
    y = dy @ w
    return y * alpha_t if alpha_t is not None else y


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, main_grad: torch.Tensor,
                 alpha_t: torch.Tensor | None = None) -> None:
    """``main_grad += dy.T @ x`` in the main-grad precision."""
    if _cuda(dy):
        _g.linear_wgrad(dy, x, main_grad, accumulate=True, alpha_t=alpha_t)
        return
    g = dy.to(main_grad.dtype).t() @ x.to(main_grad.dtype)
    if alpha_t is not None:
        g = g * alpha_t.to(main_grad.dtype)
    main_grad.add_(g)


def bias_grad(dy: torch.Tensor, main_grad: torch.Tensor) -> None:
    main_grad.add_(dy.to(main_grad.dtype).sum(0))


def swiglu_linear(x: torch.Tensor, w_gate_up: torch.Tensor, ffn: int):
    """``(silu(x Wg^T) * x Wu^T, [x Wg^T | x Wu^T])`` with ``w_gate_up = [Wg; Wu]``."""
    if _cuda(x):
        return _g.swiglu_fwd(x, w_gate_up, ffn)
    gu = x @ w_gate_up.t()
    g, u = gu[:, :ffn], gu[:, ffn:]
    return torch.nn.functional.silu(g) * u, gu


def swiglu_act(gu: torch.Tensor, ffn: int) -> torch.Tensor:
    """``silu(g) * u`` of a ``[rows, 2*ffn] = [g | u]`` tensor (the elementwise part of
    ``swiglu_linear``, for projections whose output needs a bias first)."""
    if _cuda(gu):
        h = torch.empty(gu.shape[0], ffn, device=gu.device, dtype=gu.dtype)
        lib().swiglu_fwd(gu, h)
        return h
    g, u = gu[:, :ffn], gu[:, ffn:]
    return torch.nn.functional.silu(g) * u


def swiglu_bwd(gu: torch.Tensor, dh: torch.Tensor, inplace: bool = True) -> torch.Tensor:
    """d[g|u] from the saved ``gu`` and the upstream ``dh`` (overwrites ``gu`` on CUDA)."""
    ffn = dh.shape[1]
    if _cuda(gu):
        out = gu if inplace else torch.empty_like(gu)
        lib().swiglu_bwd(gu, dh, out)
        return out
    g, u = gu[:, :ffn].float(), gu[:, ffn:].float()
    s = torch.sigmoid(g)
    d = dh.float()
    dg = d * u * s * (1 + g * (1 - s))
    du = d * g * s
    return torch.cat([dg, du], 1).to(gu.dtype)


def qkv_rope_linear(x: torch.Tensor, w_qkv: torch.Tensor, positions: torch.Tensor,
                    inv_freq: torch.Tensor, head_dim: int, rope_cols: int,
                    pos_div: int = 1) -> torch.Tensor:
    """Fused QKV projection; rotary embedding on the first ``rope_cols`` columns.

    Row ``r`` of ``x`` has position ``positions[(r // pos_div) % len(positions)]``.
    """
    if _cuda(x) and head_dim in (64, 128):
        return _g.qkv_rope_fwd(x, w_qkv, positions, inv_freq, head_dim, rope_cols,
                               pos_div=pos_div)
    y = linear(x, w_qkv)
    rope_(y, rope_cols, head_dim, positions, inv_freq, inverse=False, pos_div=pos_div)
    return y


def row_positions(rows: int, positions: torch.Tensor, pos_div: int) -> torch.Tensor:
    idx = (torch.arange(rows, device=positions.device) // pos_div) % positions.numel()
    return positions[idx]


def rope_(x: torch.Tensor, ncols: int, head_dim: int, positions: torch.Tensor,
          inv_freq: torch.Tensor, *, inverse: bool, pos_div: int = 1) -> torch.Tensor:
    """In-place rotate-half RoPE (or its inverse) on the first ``ncols`` columns."""
    if ncols == 0:
        return x
    if _cuda(x):
        pos = positions if pos_div == 1 else row_positions(x.shape[0], positions, pos_div)
        lib().rope_inplace(x, ncols, head_dim, pos.to(torch.int32).contiguous(), inv_freq,
                           inverse)
        return x
    pos = row_positions(x.shape[0], positions, pos_div).to(torch.float32)
    ang = pos[:, None] * inv_freq[None, :].float()
    cos, sin = ang.cos(), ang.sin()
    if inverse:
        sin = -sin
    half = head_dim // 2
    v = x[:, :ncols].view(x.shape[0], ncols // head_dim, head_dim)
    x1 = v[..., :half].float()
    x2 = v[..., half:].float()
    c, s = cos[:, None, :], sin[:, None, :]
    n1 = x1 * c - x2 * s
    n2 = x2 * c + x1 * s
    v[..., :half] = n1.to(x.dtype)
    v[..., half:] = n2.to(x.dtype)
    return x


# ------------------------------------------------------------------ RMSNorm
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float):
    """Returns ``(y, rstd)``; y = cast(x * rstd) * w (normalise in fp32)."""
    rows = x.numel() // x.shape[-1]
    if _cuda(x):
        y = torch.empty_like(x)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        lib().rmsnorm_fwd(x, w, y, rstd, eps)
        return y, rstd
    xf = x.float() if x.dtype != torch.float64 else x
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (xf * rstd).to(x.dtype) * w.to(x.dtype)
    return y, rstd.reshape(rows)


def rmsnorm_bwd(x: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, rstd: torch.Tensor,
                w_main_grad: torch.Tensor | None, dres: torch.Tensor | None = None
                ) -> torch.Tensor:
    """Returns dx (+ ``dres``, the residual branch gradient); accumulates dw into
    ``w_main_grad`` when given."""
    if _cuda(x):
        dx = torch.empty_like(x)
        lib().rmsnorm_bwd(x, w, dy, rstd, dx, w_main_grad, dres)
        return dx
    cd = torch.float64 if x.dtype == torch.float64 else torch.float32
    xf, dyf, wf = x.to(cd), dy.to(cd), w.to(cd)
    r = rstd.to(cd).reshape(-1, 1)
    xh = xf * r
    wg = wf * dyf
    dot = (xh * wg).mean(-1, keepdim=True)
    dx = r * (wg - xh * dot)
    if w_main_grad is not None:
        w_main_grad.add_((dyf * xh.to(x.dtype).to(cd)).sum(0).to(w_main_grad.dtype))
    if dres is not None:
        dx = dx + dres.to(cd)
    return dx.to(x.dtype)


# ------------------------------------------------------------------ embedding
def embedding(ids: torch.Tensor, w: torch.Tensor, vstart: int) -> torch.Tensor:
    """Rows of the local vocabulary shard ``[vstart, vstart + V)``; zeros elsewhere."""
    ids = ids.reshape(-1)
    if _cuda(w):
        out = torch.empty(ids.numel(), w.shape[1], device=w.device, dtype=w.dtype)
        lib().embedding_fwd(ids.contiguous(), w, vstart, out)
        return out
    local = ids - vstart
    mask = (local >= 0) & (local < w.shape[0])
    out = w[local.clamp(0, w.shape[0] - 1)]
    return out * mask[:, None].to(out.dtype)


def embedding_bwd(ids: torch.Tensor, dy: torch.Tensor, main_grad: torch.Tensor,
                  vstart: int) -> None:
    ids = ids.reshape(-1)
    if _cuda(dy):
        lib().embedding_bwd(ids.contiguous(), dy, main_grad, vstart)
        return
    local = ids - vstart
    mask = (local >= 0) & (local < main_grad.shape[0])
    main_grad.index_add_(0, local[mask], dy[mask].to(main_grad.dtype))


# ------------------------------------------------------------------ cross-entropy
def ce_local(logits: torch.Tensor, labels: torch.Tensor, write_grad: bool):
    """Single-shard CE: per-row loss (0 where label < 0); logits become
    ``softmax - onehot`` in place when ``write_grad``."""
    if _cuda(logits):
        loss_row = torch.empty(logits.shape[0], device=logits.device, dtype=torch.float32)
        lib().ce_fused(logits, labels.contiguous(), loss_row, write_grad)
        return loss_row
    return ce_finish(logits, labels, 0, ce_stats(logits, labels, 0).unsqueeze(0), write_grad)


def linear_ce(x: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, write_grad: bool):
    """LM head + single-shard cross-entropy: returns (logits, per-row loss); with
    ``write_grad`` the logits become ``softmax - onehot``. On CUDA the GEMM's epilogue
    produces the row statistics, so the cross-entropy reads the logits once."""
    if _cuda(x) and w.shape[0] % 8 == 0:
        logits, parts = _g.lm_head_ce_stats(x, w)
        loss_row = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        lib().ce_from_parts(logits, labels.contiguous(), parts, parts.shape[1], loss_row,
                            write_grad)
        return logits, loss_row
    logits = linear(x, w)
    return logits, ce_local(logits, labels, write_grad)


def ce_stats(logits: torch.Tensor, labels: torch.Tensor, vstart: int) -> torch.Tensor:
    """Per-row (max, sum exp(x - max), target logit or 0) of this vocabulary shard."""
    if _cuda(logits):
        stats = torch.empty(logits.shape[0], 3, device=logits.device, dtype=torch.float32)
        lib().ce_stats(logits, labels.contiguous(), vstart, stats)
        return stats
    cd = torch.float64 if logits.dtype == torch.float64 else torch.float32
    x = logits.to(cd)
    m = x.max(-1).values
    s = torch.exp(x - m[:, None]).sum(-1)
    local = labels - vstart
    ok = (labels >= 0) & (local >= 0) & (local < x.shape[1])
    tgt = torch.where(ok, x.gather(1, local.clamp(0, x.shape[1] - 1)[:, None])[:, 0],
                      torch.zeros_like(m))
    return torch.stack([m, s, tgt], 1)


def ce_finish(logits: torch.Tensor, labels: torch.Tensor, vstart: int, all_stats: torch.Tensor,
              write_grad: bool) -> torch.Tensor:
    """Merge ``all_stats`` ([shards, T, 3]) into per-row loss; optionally write the
    local ``softmax - onehot`` gradient into ``logits``."""
    if _cuda(logits):
        loss_row = torch.empty(logits.shape[0], device=logits.device, dtype=torch.float32)
        lib().ce_finish(logits, labels.contiguous(), vstart, all_stats.contiguous(),
                        all_stats.shape[0], loss_row, write_grad)
        return loss_row
    m = all_stats[..., 0].max(0).values
    s = (all_stats[..., 1] * torch.exp(all_stats[..., 0] - m[None])).sum(0)
    lse = m + torch.log(s)
    tgt = all_stats[..., 2].sum(0)
    valid = labels >= 0
    loss_row = torch.where(valid, lse - tgt, torch.zeros_like(lse))
    if write_grad:
        cd = all_stats.dtype
        p = torch.exp(logits.to(cd) - lse[:, None])
        local = labels - vstart
        hit = valid & (local >= 0) & (local < logits.shape[1])
        rows = torch.nonzero(hit)[:, 0]
        p[rows, local[rows]] -= 1.0
        p[~valid] = 0.0
        logits.copy_(p.to(logits.dtype))
    return loss_row.float() if loss_row.dtype != torch.float64 else loss_row


# ------------------------------------------------------------------ attention
def _pull_args(pull) -> dict:
    """``pull`` = (source address, destination tensor, flag address, epoch address): the
    attention kernel copies that ring block from the owner GPU into the destination while
    it computes (context parallelism); None = no pull."""
    if pull is None:
        return {}
    src, dst, flag, epoch = pull
    return {"pull_src": int(src), "pull_dst": dst, "pull_flag": int(flag),
            "pull_epoch": int(epoch)}


def flash_fwd(q, k, v, o, lse, scale: float, causal: bool, q_offset: int = 0,
              k_offset: int = 0, pull=None) -> None:
    """tcgen05/TMEM flash-attention forward into ``o`` ([B,S,H,D] view) and ``lse``."""
    from ._ext import status_word

    lib().flash_attn_fwd_tc(q, k, v, o, lse, scale, causal, q_offset, k_offset,
                            status_word(q.device), **_pull_args(pull))


def attention_fwd(q, k, v, *, causal: bool, q_offset: int = 0, k_offset: int = 0,
                  softmax_scale: float | None = None, pull=None):
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] (strided views). Returns (o [B,Sq,Hq,D], lse).

    ``lse`` is base-2 (log2 of the softmax denominator of scaled scores)."""
    B, Sq, Hq, D = q.shape
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    if _cuda(q):
        o = torch.empty(B, Sq, Hq, D, device=q.device, dtype=q.dtype)
        lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32)
        flash_fwd(q, k, v, o, lse, scale, causal, q_offset, k_offset, pull=pull)
        return o, lse
    o, lse = _attn_math(q, k, v, causal, q_offset, k_offset, scale)
    return o.to(q.dtype), lse


def _attn_math(q, k, v, causal, q_offset, k_offset, scale):
    cd = torch.float64 if q.dtype == torch.float64 else torch.float32
    Hq, Hkv = q.shape[2], k.shape[2]
    qf = q.to(cd).transpose(1, 2)
    kf = k.to(cd).repeat_interleave(Hq // Hkv, 2).transpose(1, 2)
    vf = v.to(cd).repeat_interleave(Hq // Hkv, 2).transpose(1, 2)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        qp = torch.arange(q.shape[1]) + q_offset
        kp = torch.arange(k.shape[1]) + k_offset
        s = s.masked_fill((kp[None, :] > qp[:, None]).to(s.device), float("-inf"))
    lse_e = torch.logsumexp(s, -1)
    p = torch.exp(s - lse_e[..., None]).nan_to_num(0.0)
    o = (p @ vf).transpose(1, 2)
    return o, lse_e / math.log(2.0)


def attention_bwd(q, k, v, o, do, lse, dq, dk, dv, *, causal: bool, q_offset: int = 0,
                  k_offset: int = 0, softmax_scale: float | None = None,
                  q_pos: torch.Tensor | None = None, k_pos: torch.Tensor | None = None,
                  inv_freq: torch.Tensor | None = None, pull=None) -> None:
    """Writes dq/dk/dv (strided views). With ``q_pos``/``k_pos`` the inverse RoPE
    is applied to dq/dk on the way out (gradients w.r.t. pre-rotation q/k)."""
    B, Sq, Hq, D = q.shape
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    if _cuda(q):
        from ._ext import status_word
        from .deterministic import is_deterministic

        n = B * Sq * Hq * D
        delta = torch.empty(B * Hq * Sq, device=q.device, dtype=torch.float32)
        dq_acc = torch.empty(n, device=q.device, dtype=torch.float32)
        L = lib()
        L.flash_attn_bwd_prep(o, do, delta, dq_acc)
        k_cs = None
        if k_pos is not None and inv_freq is not None:
            from .gemm import rope_table

            k_cs = rope_table(k_pos, inv_freq)
        # Deterministic mode: one zeroed dQ slot per 128-key block (blocks a causal mask
        # skips stay zero), summed in key-block order into the zeroed accumulator.
        slots = (torch.zeros((k.shape[1] + 127) // 128, n, device=q.device, dtype=torch.float32)
                 if is_deterministic() else None)
        L.flash_attn_bwd_tc_kv(q, k, v, do, lse, delta, dq_acc if slots is None else slots,
                               dk, dv, scale, causal, q_offset, k_offset, k_pos, inv_freq,
                               status_word(q.device), **_pull_args(pull), k_cs=k_cs,
                               dq_slot_stride=0 if slots is None else n)
        if slots is not None:
            L.slots_sum(slots, dq_acc, True)
        L.flash_attn_bwd_dq_convert(dq_acc, dq, q_pos, inv_freq)
        return
    # Explicit flash-attention backward using the given (global) log-sum-exp, so a
    # partial key block (ring attention) gets its share of the global softmax.
    cd = torch.float64 if q.dtype == torch.float64 else torch.float32
    Hkv = k.shape[2]
    rep = Hq // Hkv
    qf = q.to(cd).transpose(1, 2)                                   # [B, Hq, Sq, D]
    kf = k.to(cd).repeat_interleave(rep, 2).transpose(1, 2)        # [B, Hq, Sk, D]
    vf = v.to(cd).repeat_interleave(rep, 2).transpose(1, 2)
    of = o.to(cd).transpose(1, 2)
    dof = do.to(cd).transpose(1, 2)
    s = (qf @ kf.transpose(-1, -2)) * scale
    p = torch.exp2(s * math.log2(math.e) - lse.to(cd)[..., None])
    if causal:
        qp = torch.arange(q.shape[1]) + q_offset
        kp = torch.arange(k.shape[1]) + k_offset
        p = p.masked_fill((kp[None, :] > qp[:, None]).to(p.device), 0.0)
    p = p.nan_to_num(0.0)
    dvf = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    delta = (dof * of).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dqf = (ds @ kf) * scale
    dkf = (ds.transpose(-1, -2) @ qf) * scale
    gq = dqf.transpose(1, 2)
    gk = dkf.view(B, Hkv, rep, -1, D).sum(2).transpose(1, 2)
    gv = dvf.view(B, Hkv, rep, -1, D).sum(2).transpose(1, 2)
    for dst, src, pos in ((dq, gq, q_pos), (dk, gk, k_pos), (dv, gv, None)):
        if pos is not None:
            flat = src.to(dst.dtype).reshape(B * src.shape[1], -1).clone()
            # rows are (b, s) ordered: position index = s
            rope_(flat, flat.shape[1], D, pos, inv_freq, inverse=True, pos_div=1)
            dst.copy_(flat.view_as(src))
        else:
            dst.copy_(src)


# ------------------------------------------------------------------ optimizer pieces
def adamw_(p, g, m, v, p_low, *, lr, beta1, beta2, eps, weight_decay, step,
           grad_scale: torch.Tensor | None = None, lr_t: torch.Tensor | None = None) -> None:
    """torch.optim.AdamW update over flat fp32 buffers (optionally writes a low-precision copy)."""
    if p.is_cuda:
        lib().adamw_step(p, g, m, v, p_low, lr, beta1, beta2, eps, weight_decay, step,
                         grad_scale, lr_t)
        return
    lr_v = float(lr_t.item()) if lr_t is not None else lr
    gr = g if grad_scale is None else g * grad_scale
    p.mul_(1 - lr_v * weight_decay)
    m.mul_(beta1).add_(gr, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(gr, gr, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr_v / bc1)
    if p_low is not None:
        p_low.copy_(p)


def sumsq(x: torch.Tensor) -> torch.Tensor:
    """Sum of squares as a 0-d fp32 (fp64 on CPU for fp64 input) device tensor."""
    if x.numel() == 0:
        return torch.zeros((), device=x.device, dtype=torch.float32)
    if x.is_cuda and x.dtype == torch.float32 and x.is_contiguous():
        return lib().sumsq_partials(x).sum()
    return x.double().pow(2).sum().to(torch.float32 if x.dtype != torch.float64 else x.dtype)
