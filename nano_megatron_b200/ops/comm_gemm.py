"""Fused tensor-parallel GEMM + collective ops over a :class:`SymmetricWorkspace`.

* ``gemm_reduce_scatter``: ``out[R, N] = sum_r (A_r B_r^T)[rows of this rank] (+ residual)``
  -- the row-parallel projection under sequence parallelism (out_proj / down_proj
  forward, QKV / gate-up dgrad). One tcgen05 GEMM whose epilogue stores each bf16
  partial tile into its owner's staging slot over NVLink, then a flag-gated
  reduce on the owner that also adds the residual.
* ``allgather_gemm``: ``out[M, N] = epilogue(concat_r(X_r) B^T)`` -- the
  column-parallel projection under sequence parallelism (QKV with RoPE, gate|up
  with SwiGLU, out/down dgrad). The local shard is published into the symmetric
  buffer and signalled; the GEMM's TMA producer reads each peer's rows straight
  from that peer's buffer once its flag arrives, own rows first, and the gathered
  input is written to a local tensor for the backward pass.

Each op is split into ``issue`` / ``finish`` phases so single-GPU tests can run
emulated ranks phase by phase; the public functions run both.
"""

from __future__ import annotations

import os

import torch

from nano_megatron_b200.distributed.symmetric import CH_AG, CH_CE, CH_EMB, CH_RS

from ._ext import lib

EPI = {"bf16": 0, "rope": 3, "swiglu": 2, "ce_stats": 5}

# GEMM -> reduce-scatter with this rank's rows reduced in the GEMM's own epilogue (per-tile
# flags) instead of a second kernel. Off by default: on 2 x B200 at the 311M out_proj shape
# (32768 x 1024 x 512, TP2) it measured 122 us against 110 us for the two-pass path
# (``python -m nano_megatron_b200.ops.bench_comm --case tp``); the per-tile release of the
# peer tiles serialises the epilogue. NMB_RS_IN_KERNEL=1 selects it.
RS_IN_KERNEL = os.environ.get("NMB_RS_IN_KERNEL", "0") == "1"


def rs_issue(ws, a: torch.Tensor, b: torch.Tensor, *, b_mn: bool = False,
             n_out: int | None = None, alpha_t: torch.Tensor | None = None,
             out: torch.Tensor | None = None, residual: torch.Tensor | None = None
             ) -> tuple[int, int, bool]:
    """GEMM with the peer epilogue + signal. Returns (rows_per_rank, n_out, reduced).
    ``alpha_t``: optional fp32 device scalar multiplying the product. With ``out`` (and a
    real multi-GPU workspace) the kernel also reduces this rank's rows into ``out``
    (+ ``residual``) in its epilogue and ``reduced`` is True; otherwise ``rs_finish``
    does the reduction in a second kernel."""
    M = a.shape[0]
    if M % ws.size:
        raise ValueError(f"rows {M} not divisible by TP size {ws.size}")
    rows = M // ws.size
    n = n_out if n_out is not None else (b.shape[1] if b_mn else b.shape[0])
    ws.check_rs(rows, n)
    inplace = out is not None and RS_IN_KERNEL and not getattr(ws, "emulated", False)
    lib().gemm_tc_rs(a, False, b, b_mn, [ws.rs_staging(r, 0) for r in range(ws.size)],
                     [ws.rs_staging(r, 1) for r in range(ws.size)], rows, n, ws.rank,
                     ws.epoch_ptr(CH_RS), ws.status, alpha_t,
                     out if inplace else None, residual if inplace else None,
                     [ws.rs_tile_flags(r) for r in range(ws.size)] if inplace else [])
    lib().peer_signal(ws.signal_targets(CH_RS), ws.epoch_ptr(CH_RS))
    return rows, n, inplace


def rs_finish(ws, out: torch.Tensor, residual: torch.Tensor | None = None) -> None:
    lib().rs_reduce(ws.rs_staging(ws.rank, 0), ws.rs_staging(ws.rank, 1), ws.size, out, residual,
                    ws.flags(ws.rank, CH_RS), ws.epoch_ptr(CH_RS), ws.status)


def gemm_reduce_scatter(ws, a: torch.Tensor, b: torch.Tensor, *, b_mn: bool = False,
                        residual: torch.Tensor | None = None,
                        out: torch.Tensor | None = None,
                        alpha_t: torch.Tensor | None = None) -> torch.Tensor:
    M = a.shape[0]
    n = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty(M // ws.size, n, device=a.device, dtype=torch.bfloat16)
    if residual is not None and (residual.stride(-1) != 1 or residual.stride(0) % 8):
        residual = residual.contiguous()
    _, _, reduced = rs_issue(ws, a, b, b_mn=b_mn, alpha_t=alpha_t, out=out, residual=residual)
    if not reduced:
        rs_finish(ws, out, residual)
    return out


def ag_issue(ws, x_local: torch.Tensor, channel: int = CH_AG) -> None:
    """Publish this rank's shard into its symmetric slot and signal every rank."""
    R, K = x_local.shape
    ws.check_ag(R, K)
    lib().ag_publish(x_local, ws.ag_shard(ws.rank, 0), ws.ag_shard(ws.rank, 1),
                     ws.epoch_ptr(channel))
    lib().peer_signal(ws.signal_targets(channel), ws.epoch_ptr(channel))


def ag_finish(ws, x_local: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *,
              b_mn: bool = False, epi: str = "bf16", xfull: torch.Tensor | None = None,
              aux: torch.Tensor | None = None, swiglu_up_row: int = 0,
              positions: torch.Tensor | None = None, inv_freq: torch.Tensor | None = None,
              head_dim: int = 0, rope_cols: int = 0, pos_div: int = 1,
              channel: int = CH_AG, ce_part: torch.Tensor | None = None) -> None:
    R, K = x_local.shape
    table = None
    if epi == "rope":
        from .gemm import rope_table

        table = rope_table(positions, inv_freq, torch.bfloat16)
    ready = ws.gather_ready[channel] if out.shape[0] // 128 <= ws.gather_ready.shape[1] \
        else None
    lib().gemm_tc_ag(x_local, [ws.ag_shard(r, 0) for r in range(ws.size)],
                     [ws.ag_shard(r, 1) for r in range(ws.size)], K, b, b_mn, out, EPI[epi],
                     xfull, aux, swiglu_up_row, positions, inv_freq, head_dim, rope_cols,
                     pos_div, ws.rank, ws.flags(ws.rank, channel), ws.epoch_ptr(channel),
                     ws.status, table, ready, ce_part)


def allgather_gemm(ws, x_local: torch.Tensor, b: torch.Tensor, *, b_mn: bool = False,
                   epi: str = "bf16", n_out: int | None = None, store_gathered: bool = True,
                   **kw) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Returns (out [TP*R, N], gathered input [TP*R, K] or None)."""
    R, K = x_local.shape
    M = R * ws.size
    n = n_out if n_out is not None else (b.shape[1] if b_mn else b.shape[0])
    out = torch.empty(M, n, device=x_local.device, dtype=torch.bfloat16)
    xfull = torch.empty(M, K, device=x_local.device, dtype=torch.bfloat16) \
        if store_gathered else None
    ag_issue(ws, x_local)
    ag_finish(ws, x_local, b, out, b_mn=b_mn, epi=epi, xfull=xfull, **kw)
    return out, xfull


# ---------------------------------------------------------------- embedding (C3)
def embedding_issue(ws, ids: torch.Tensor, weight: torch.Tensor, vstart: int) -> int:
    """Store the rows of this vocabulary shard into the sequence owners' slots + signal.
    ``ids``: every token of the TP group's block, sequence-major. Returns rows per rank."""
    T = ids.numel()
    if T % ws.size:
        raise ValueError(f"{T} tokens not divisible by TP size {ws.size}")
    R = T // ws.size
    ws.check_emb(R, weight.shape[1])
    lib().tp_embedding_scatter(ids, weight, vstart, R, [ws.emb_slot(r, 0) for r in range(ws.size)],
                               [ws.emb_slot(r, 1) for r in range(ws.size)], ws.epoch_ptr(CH_EMB))
    lib().peer_signal(ws.signal_targets(CH_EMB), ws.epoch_ptr(CH_EMB))
    return R


def embedding_finish(ws, out: torch.Tensor) -> None:
    lib().tp_embedding_collect(ws.emb_slot(ws.rank, 0), ws.emb_slot(ws.rank, 1), out, ws.size,
                               ws.flags(ws.rank, CH_EMB), ws.epoch_ptr(CH_EMB), ws.status)


def embedding_lookup_scatter(ws, ids: torch.Tensor, weight: torch.Tensor,
                             vstart: int) -> torch.Tensor:
    """Vocabulary-parallel lookup fused with the sequence-parallel reduce-scatter: this
    rank's [T / TP, H] rows of the embedding output."""
    R = embedding_issue(ws, ids, weight, vstart)
    out = torch.empty(R, weight.shape[1], device=weight.device, dtype=weight.dtype)
    embedding_finish(ws, out)
    return out


def embedding_bwd_finish(ws, ids: torch.Tensor, dy_local: torch.Tensor, grad: torch.Tensor,
                         vstart: int) -> None:
    R, H = dy_local.shape
    lib().tp_embedding_bwd_gather(ids, [ws.ag_shard(r, 0) for r in range(ws.size)],
                                  [ws.ag_shard(r, 1) for r in range(ws.size)], R, H, grad,
                                  vstart, ws.flags(ws.rank, CH_AG), ws.epoch_ptr(CH_AG),
                                  ws.status)


def embedding_backward_gather(ws, ids: torch.Tensor, dy_local: torch.Tensor,
                              grad: torch.Tensor, vstart: int) -> None:
    """Embedding backward fused with the sequence-parallel all-gather of dY: publish this
    rank's dY rows, then add every token of this vocabulary shard into ``grad`` (fp32)
    reading its dY row from the owning rank."""
    ag_issue(ws, dy_local)
    embedding_bwd_finish(ws, ids, dy_local, grad, vstart)


# ---------------------------------------------------------------- cross-entropy (C6)
def ce_issue(ws, logits: torch.Tensor, labels: torch.Tensor, vstart: int,
             parts: torch.Tensor | None = None) -> None:
    """Store this rank's per-row (max, sum exp, target logit) into every TP rank's slot +
    signal. With ``parts`` (the LM-head GEMM epilogue's per-tile statistics) only the target
    logits are read back from ``logits``."""
    ws.check_ce(logits.shape[0])
    slots = ([ws.ce_slot(r, 0) for r in range(ws.size)], [ws.ce_slot(r, 1) for r in range(ws.size)])
    if parts is not None:
        lib().tp_ce_parts_scatter(logits, labels, vstart, parts, parts.shape[1], ws.rank, *slots,
                                  ws.epoch_ptr(CH_CE))
    else:
        lib().tp_ce_stats_scatter(logits, labels, vstart, ws.rank, *slots, ws.epoch_ptr(CH_CE))
    lib().peer_signal(ws.signal_targets(CH_CE), ws.epoch_ptr(CH_CE))


def ce_finish(ws, logits: torch.Tensor, labels: torch.Tensor, vstart: int,
              write_grad: bool) -> torch.Tensor:
    loss_row = torch.empty(logits.shape[0], device=logits.device, dtype=torch.float32)
    lib().tp_ce_finish_gather(logits, labels, vstart, ws.ce_slot(ws.rank, 0),
                              ws.ce_slot(ws.rank, 1), ws.size, loss_row, write_grad,
                              ws.flags(ws.rank, CH_CE), ws.epoch_ptr(CH_CE), ws.status)
    return loss_row


def vocab_parallel_ce_rows(ws, logits: torch.Tensor, labels: torch.Tensor, vstart: int,
                           write_grad: bool, parts: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row loss of the vocabulary-parallel cross-entropy; the row statistics travel by
    peer stores + flag instead of a collective. With ``write_grad`` the local logits are
    overwritten by d loss_row / d logits."""
    ce_issue(ws, logits, labels, vstart, parts)
    return ce_finish(ws, logits, labels, vstart, write_grad)
