"""Fused per-block autograd functions of the GPT training path.

One ``torch.autograd.Function`` per transformer sub-block keeps the Python
overhead per layer to two calls and lets each block choose its own kernel
schedule:

* attention block: RMSNorm -> [SP all-gather] -> QKV GEMM with RoPE epilogue
  -> causal flash attention (local or context-parallel core) -> out-proj GEMM
  with the residual add in its epilogue -> [SP reduce-scatter / TP all-reduce];
* MLP block: RMSNorm -> [SP all-gather] -> gate|up GEMM with SwiGLU epilogue
  -> down GEMM with residual epilogue -> [SP reduce-scatter / TP all-reduce];
* embedding (vocab-parallel gather + TP reduction) and LM head (final norm,
  logits GEMM, vocab-parallel cross-entropy whose gradient overwrites the
  logits in place, so no fp32 logits or softmax copy is ever stored).

Under sequence parallelism with a symmetric workspace attached (CUDA, TP > 1),
the SP collectives are fused into the GEMMs over NVLink: the norm output's
all-gather into the QKV / gate|up GEMM (TMA loads from the peers' shards, the
gathered input kept for the weight gradient), the out/down projection's
reduce-scatter into its GEMM epilogue (plus the residual add), and in the
backward pass the dY all-gather into the dgrad GEMM and the dX reduce-scatter
into the QKV / gate|up dgrad GEMM (:mod:`nano_megatron_b200.ops.comm_gemm`).

Weight gradients are accumulated straight into each parameter's fp32
``main_grad`` (a view of the data-parallel gradient buffer) by the
weight-gradient GEMM epilogue; autograd returns ``None`` for parameters.
Activations are sequence-major ``[S, B, H]`` flattened to ``[S*B, H]``; under
sequence parallelism each TP rank holds a contiguous block of S/TP rows.

The reference computes the same math module by module
(src/nano_megatron/models/gpt/layer.py:91-137, attention.py:153-209,
mlp.py:42-78, model.py:171-250).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from nano_megatron_b200.ops import functional as F
from nano_megatron_b200.ops import comm_gemm as CG
from nano_megatron_b200.tensor_parallel.comm import all_gather_dim0, all_reduce, reduce_scatter_dim0
from nano_megatron_b200.tensor_parallel.cross_entropy import vocab_parallel_ce_rows


def main_grad_of(p: torch.Tensor) -> torch.Tensor:
    """The fp32 gradient accumulator of ``p`` (created on first use if no buffer owns it)."""
    g = getattr(p, "main_grad", None)
    if g is None:
        dt = torch.float64 if p.dtype == torch.float64 else torch.float32
        g = torch.zeros(p.shape, dtype=dt, device=p.device)
        p.main_grad = g
    return g


def _contiguous_run(tensors: list[torch.Tensor]) -> bool:
    ptr = tensors[0].data_ptr()
    for t in tensors:
        if not t.is_contiguous() or t.data_ptr() != ptr:
            return False
        ptr += t.numel() * t.element_size()
    return True


def fused_rows(params: list[torch.Tensor]) -> torch.Tensor:
    """Row-concatenation of 2-D weights: a zero-copy view when they are adjacent in memory."""
    if _contiguous_run(params):
        rows = sum(p.shape[0] for p in params)
        return torch.as_strided(params[0].detach(), (rows, params[0].shape[1]),
                                (params[0].shape[1], 1))
    return torch.cat([p.detach() for p in params], 0)


class FusedGrad:
    """Row-concatenated main-grad target for several parameters.

    If their accumulators are adjacent it is a view; otherwise a scratch buffer
    that :meth:`flush` adds back into each parameter's accumulator."""

    def __init__(self, params: list[torch.Tensor]):
        self.params = params
        grads = [main_grad_of(p) for p in params]
        if _contiguous_run(grads):
            rows = sum(g.shape[0] for g in grads)
            self.target = torch.as_strided(grads[0], (rows,) + tuple(grads[0].shape[1:]),
                                           grads[0].stride())
            self.scratch = False
        else:
            self.target = torch.zeros((sum(g.shape[0] for g in grads),) + tuple(grads[0].shape[1:]),
                                      dtype=grads[0].dtype, device=grads[0].device)
            self.scratch = True

    def flush(self) -> None:
        if not self.scratch:
            return
        off = 0
        for p in self.params:
            n = p.shape[0]
            main_grad_of(p).add_(self.target[off:off + n])
            off += n


@dataclass
class TPInfo:
    group: object | None
    size: int
    sequence_parallel: bool
    workspace: object | None = None   # SymmetricWorkspace for the fused SP collectives

    def fused(self, x: torch.Tensor) -> bool:
        """Use the fused AG->GEMM / GEMM->RS kernels for this local row block."""
        return x.is_cuda and self.fused_rows(x.shape[0])

    def fused_rows(self, rows: int) -> bool:
        return (self.workspace is not None and self.sequence_parallel and self.size > 1 and
                rows % 128 == 0)

    def gather(self, x):
        return all_gather_dim0(x, self.group) if self.sequence_parallel and self.size > 1 else x

    def reduce_out(self, y):
        """Reduction after a row-parallel GEMM (forward)."""
        if self.size == 1:
            return y
        return reduce_scatter_dim0(y, self.group) if self.sequence_parallel else \
            all_reduce(y, self.group)

    def reduce_in_grad(self, dx):
        """Reduction of the input gradient of a column-parallel GEMM (backward)."""
        if self.size == 1:
            return dx
        return reduce_scatter_dim0(dx, self.group) if self.sequence_parallel else \
            all_reduce(dx, self.group)


@dataclass
class MicrobatchInfo:
    """Per-microbatch runtime facts shared by all blocks of one forward."""

    batch: int                 # B
    seq: int                   # S_local (this CP rank's sequence length, before SP)
    positions: torch.Tensor    # int32 [S_local], absolute positions of local tokens
    cp_chunks: tuple = ()      # ((start_row, length, position_offset), ...) of local chunks
    microbatch_index: int = 0
    extra: dict = field(default_factory=dict)


# ---------------------------------------------------------------- attention core
class LocalAttentionCore:
    """Causal flash attention over the local sequence (no context parallelism)."""

    applies_inverse_rope = True

    def forward(self, q, k, v, o, mb: MicrobatchInfo):
        o_bs = o.transpose(0, 1)
        B, S, Hq, D = o_bs.shape
        lse = torch.empty(B, Hq, S, device=q.device, dtype=torch.float32)
        if q.is_cuda:
            F.flash_fwd(q, k, v, o_bs, lse, D ** -0.5, True)
        else:
            out, lse2 = F.attention_fwd(q, k, v, causal=True)
            o_bs.copy_(out)
            lse.copy_(lse2)
        return lse

    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb: MicrobatchInfo, inv_freq):
        F.attention_bwd(q, k, v, o.transpose(0, 1), do, lse, dq, dk, dv, causal=True,
                        q_pos=mb.positions, k_pos=mb.positions, inv_freq=inv_freq)


def _split_qkv(qkv2d: torch.Tensor, S: int, B: int, hq: int, hkv: int, D: int):
    v4 = qkv2d.view(S, B, hq + 2 * hkv, D)
    q = v4[:, :, :hq].transpose(0, 1)
    k = v4[:, :, hq:hq + hkv].transpose(0, 1)
    v = v4[:, :, hq + hkv:].transpose(0, 1)
    return q, k, v


@dataclass
class AttnSpec:
    hidden: int
    heads: int          # local query heads
    kv_heads: int       # local kv heads
    head_dim: int
    eps: float
    tp: TPInfo
    core: object
    dropout: float = 0.0


class AttentionBlockFn(torch.autograd.Function):
    """h_out = h + out_proj(attn(rope(qkv(norm(h))))) with TP/SP collectives."""

    @staticmethod
    def forward(ctx, h, w_norm, w_q, w_k, w_v, w_out, b_out, spec: AttnSpec, mb: MicrobatchInfo,
                inv_freq, dropout_fn, b_qkv=None):
        """``b_qkv``: the (q, k, v) column-parallel biases when the model has biases; they
        are added before the rotary embedding, as in the reference's attention."""
        H = spec.hidden
        h2 = h.reshape(-1, H)
        xn, rstd = F.rmsnorm(h2, w_norm, spec.eps)
        w_qkv = fused_rows([w_q, w_k, w_v])
        D, hq, hkv = spec.head_dim, spec.heads, spec.kv_heads
        fused = spec.tp.fused(xn) and D in (64, 128) and b_qkv is None
        if fused:
            qkv, xg = CG.allgather_gemm(spec.tp.workspace, xn, w_qkv, epi="rope",
                                        positions=mb.positions, inv_freq=inv_freq, head_dim=D,
                                        rope_cols=(hq + hkv) * D, pos_div=mb.batch)
        elif b_qkv is None:
            xg = spec.tp.gather(xn)
            qkv = F.qkv_rope_linear(xg, w_qkv, mb.positions, inv_freq, D, (hq + hkv) * D,
                                    pos_div=mb.batch)
        else:
            xg = spec.tp.gather(xn)
            qkv = F.linear(xg, w_qkv)
            qkv += torch.cat([b.detach() for b in b_qkv]).to(qkv.dtype)
            F.rope_(qkv, (hq + hkv) * D, D, mb.positions, inv_freq, inverse=False,
                    pos_div=mb.batch)
        q, k, v = _split_qkv(qkv, mb.seq, mb.batch, hq, hkv, D)
        o = torch.empty(mb.seq, mb.batch, hq, D, device=h.device, dtype=qkv.dtype)
        lse = spec.core.forward(q, k, v, o, mb)
        ctx2 = o.view(mb.seq * mb.batch, hq * D)
        fuse_residual = spec.tp.size == 1 and b_out is None and dropout_fn is None
        if fuse_residual:
            out = F.linear(ctx2, w_out.detach(), residual=h2)
        elif fused and b_out is None and dropout_fn is None:
            out = CG.gemm_reduce_scatter(spec.tp.workspace, ctx2, w_out.detach(), residual=h2)
        else:
            y = spec.tp.reduce_out(F.linear(ctx2, w_out.detach()))
            if b_out is not None:
                y = y + b_out.detach()
            if dropout_fn is not None:
                y = dropout_fn(y)
            out = h2 + y
        ctx.spec, ctx.mb, ctx.inv_freq = spec, mb, inv_freq
        ctx.layer = mb.extra.get("layer")
        ctx.params = (w_norm, w_q, w_k, w_v, w_out, b_out)
        ctx.b_qkv = b_qkv
        ctx.dropout_fn = dropout_fn
        ctx.save_for_backward(h2, rstd, xg, qkv, o, lse)
        return out.view(h.shape)

    @staticmethod
    def backward(ctx, dout):
        spec, mb = ctx.spec, ctx.mb
        h2, rstd, xg, qkv, o, lse = ctx.saved_tensors
        w_norm, w_q, w_k, w_v, w_out, b_out = ctx.params
        D, hq, hkv = spec.head_dim, spec.heads, spec.kv_heads
        dh = dout.reshape(h2.shape).contiguous()
        dy = dh
        if ctx.dropout_fn is not None:
            dy = ctx.dropout_fn.backward(dy)
        if b_out is not None:
            F.bias_grad(dy, main_grad_of(b_out))
        ctx2 = o.view(mb.seq * mb.batch, hq * D)
        fused = spec.tp.fused(dy)
        if fused:
            d_ctx, dyg = CG.allgather_gemm(spec.tp.workspace, dy, w_out.detach(), b_mn=True)
        else:
            dyg = spec.tp.gather(dy)
            d_ctx = F.linear_dgrad(dyg, w_out.detach())
        F.linear_wgrad(dyg, ctx2, main_grad_of(w_out))
        q, k, v = _split_qkv(qkv, mb.seq, mb.batch, hq, hkv, D)
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = _split_qkv(dqkv, mb.seq, mb.batch, hq, hkv, D)
        do = d_ctx.view(mb.seq, mb.batch, hq, D).transpose(0, 1)
        mb.extra["layer"] = ctx.layer
        spec.core.backward(q, k, v, o, do, lse, dq, dk, dv, mb, ctx.inv_freq)
        del d_ctx
        if not getattr(spec.core, "applies_inverse_rope", True):
            F.rope_(dqkv, (hq + hkv) * D, D, mb.positions, ctx.inv_freq, inverse=True,
                    pos_div=mb.batch)
        if ctx.b_qkv is not None:
            gb = FusedGrad(list(ctx.b_qkv))
            F.bias_grad(dqkv, gb.target)
            gb.flush()
        w_qkv = fused_rows([w_q, w_k, w_v])
        if fused:
            dxn = CG.gemm_reduce_scatter(spec.tp.workspace, dqkv, w_qkv, b_mn=True)
        else:
            dxn = spec.tp.reduce_in_grad(F.linear_dgrad(dqkv, w_qkv))
        g = FusedGrad([w_q, w_k, w_v])
        F.linear_wgrad(dqkv, xg, g.target)
        g.flush()
        dh_in = F.rmsnorm_bwd(h2, w_norm.detach(), dxn, rstd, main_grad_of(w_norm), dres=dh)
        return (dh_in.view(dout.shape), None, None, None, None, None, None, None, None, None, None,
                None)


@dataclass
class MLPSpec:
    hidden: int
    ffn: int            # local FFN width (F / TP)
    eps: float
    tp: TPInfo


class MLPBlockFn(torch.autograd.Function):
    """h_out = h + down(silu(gate(norm(h))) * up(norm(h))) with TP/SP collectives."""

    @staticmethod
    def forward(ctx, h, w_norm, w_gate, w_up, w_down, b_down, spec: MLPSpec, dropout_fn,
                b_gu=None):
        """``b_gu``: the (gate, up) column-parallel biases when the model has biases; they
        are added before the SwiGLU activation."""
        H = spec.hidden
        h2 = h.reshape(-1, H)
        xn, rstd = F.rmsnorm(h2, w_norm, spec.eps)
        w_gu = fused_rows([w_gate, w_up])
        # any local FFN width with 16-byte rows: the SwiGLU epilogue predicates the last
        # (partial) tile, e.g. 1368 = 2736 / TP2 for the 311M model
        fused = spec.tp.fused(xn) and spec.ffn % 8 == 0 and b_gu is None
        if fused:
            gu = torch.empty(xn.shape[0] * spec.tp.size, 2 * spec.ffn, device=xn.device,
                             dtype=xn.dtype)
            hmid, xg = CG.allgather_gemm(spec.tp.workspace, xn, w_gu, epi="swiglu",
                                         n_out=spec.ffn, aux=gu, swiglu_up_row=spec.ffn)
        elif b_gu is None:
            xg = spec.tp.gather(xn)
            hmid, gu = F.swiglu_linear(xg, w_gu, spec.ffn)
        else:
            xg = spec.tp.gather(xn)
            gu = F.linear(xg, w_gu)
            gu += torch.cat([b.detach() for b in b_gu]).to(gu.dtype)
            hmid = F.swiglu_act(gu, spec.ffn)
        fuse_residual = spec.tp.size == 1 and b_down is None and dropout_fn is None
        if fuse_residual:
            out = F.linear(hmid, w_down.detach(), residual=h2)
        elif fused and b_down is None and dropout_fn is None:
            out = CG.gemm_reduce_scatter(spec.tp.workspace, hmid, w_down.detach(), residual=h2)
        else:
            y = spec.tp.reduce_out(F.linear(hmid, w_down.detach()))
            if b_down is not None:
                y = y + b_down.detach()
            if dropout_fn is not None:
                y = dropout_fn(y)
            out = h2 + y
        ctx.spec = spec
        ctx.params = (w_norm, w_gate, w_up, w_down, b_down)
        ctx.b_gu = b_gu
        ctx.dropout_fn = dropout_fn
        ctx.save_for_backward(h2, rstd, xg, gu, hmid)
        return out.view(h.shape)

    @staticmethod
    def backward(ctx, dout):
        spec = ctx.spec
        h2, rstd, xg, gu, hmid = ctx.saved_tensors
        w_norm, w_gate, w_up, w_down, b_down = ctx.params
        dh = dout.reshape(h2.shape).contiguous()
        dy = dh
        if ctx.dropout_fn is not None:
            dy = ctx.dropout_fn.backward(dy)
        if b_down is not None:
            F.bias_grad(dy, main_grad_of(b_down))
        fused = spec.tp.fused(dy) and spec.ffn % 8 == 0
        if fused:
            dmid, dyg = CG.allgather_gemm(spec.tp.workspace, dy, w_down.detach(), b_mn=True)
        else:
            dyg = spec.tp.gather(dy)
            dmid = F.linear_dgrad(dyg, w_down.detach())
        F.linear_wgrad(dyg, hmid, main_grad_of(w_down))
        dgu = F.swiglu_bwd(gu, dmid, inplace=True)
        del dmid
        if ctx.b_gu is not None:
            gb = FusedGrad(list(ctx.b_gu))
            F.bias_grad(dgu, gb.target)
            gb.flush()
        w_gu = fused_rows([w_gate, w_up])
        if fused:
            dxn = CG.gemm_reduce_scatter(spec.tp.workspace, dgu, w_gu, b_mn=True)
        else:
            dxn = spec.tp.reduce_in_grad(F.linear_dgrad(dgu, w_gu))
        g = FusedGrad([w_gate, w_up])
        F.linear_wgrad(dgu, xg, g.target)
        g.flush()
        dh_in = F.rmsnorm_bwd(h2, w_norm.detach(), dxn, rstd, main_grad_of(w_norm), dres=dh)
        return dh_in.view(dout.shape), None, None, None, None, None, None, None, None


class EmbeddingFn(torch.autograd.Function):
    """Vocab-parallel lookup of sequence-major ids, summed over TP (RS under SP).

    With the fused TP workspace the reduce-scatter is a selection done by the lookup
    itself (each rank stores only the rows of its vocabulary shard into the sequence
    owner's slot) and the backward reads the dY rows of its shard straight from their
    owners (:func:`nano_megatron_b200.ops.comm_gemm.embedding_lookup_scatter`)."""

    @staticmethod
    def forward(ctx, ids, weight, vstart: int, tp: TPInfo):
        fused = tp.fused_rows(ids.numel() // max(tp.size, 1)) and weight.shape[1] % 8 == 0
        if fused:
            out = CG.embedding_lookup_scatter(tp.workspace, ids, weight.detach(), vstart)
        else:
            out = F.embedding(ids, weight.detach(), vstart)
            out = tp.reduce_out(out)
        ctx.vstart, ctx.tp, ctx.weight, ctx.fused = vstart, tp, weight, fused
        ctx.save_for_backward(ids)
        return out

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        if ctx.fused:
            CG.embedding_backward_gather(ctx.tp.workspace, ids, dy2, main_grad_of(ctx.weight),
                                         ctx.vstart)
        else:
            dyg = ctx.tp.gather(dy2)
            F.embedding_bwd(ids, dyg, main_grad_of(ctx.weight), ctx.vstart)
        return None, None, None, None


class HeadLossFn(torch.autograd.Function):
    """Final RMSNorm + vocab-parallel logits + cross-entropy (mean over valid tokens).

    The CE kernel replaces the logits by ``softmax - onehot`` in place; backward
    scales it by ``grad / count`` inside the dgrad/wgrad GEMM epilogues."""

    @staticmethod
    def forward(ctx, h, w_norm, w_lm, labels, eps: float, tp: TPInfo):
        H = h.shape[-1]
        h2 = h.reshape(-1, H)
        xn, rstd = F.rmsnorm(h2, w_norm.detach(), eps)
        fused = tp.fused(xn) and w_lm.shape[0] % 8 == 0
        if fused:
            # AG -> LM-head GEMM whose epilogue also writes each row's per-tile (max, sum exp),
            # then the row statistics exchanged by peer stores + flag
            from nano_megatron_b200.ops.gemm import ce_parts_per_row

            parts = torch.empty(xn.shape[0] * tp.size, ce_parts_per_row(w_lm.shape[0]), 2,
                                device=xn.device, dtype=torch.float32)
            logits, xg = CG.allgather_gemm(tp.workspace, xn, w_lm.detach(), epi="ce_stats",
                                           ce_part=parts)
            rows = CG.vocab_parallel_ce_rows(tp.workspace, logits, labels,
                                             tp.workspace.rank * w_lm.shape[0], write_grad=True,
                                             parts=parts)
        elif tp.size == 1:
            # LM head + cross-entropy: the GEMM epilogue writes the row statistics
            xg = xn
            logits, rows = F.linear_ce(xg, w_lm.detach(), labels, write_grad=True)
        else:
            xg = tp.gather(xn)
            logits = F.linear(xg, w_lm.detach())
            rows = vocab_parallel_ce_rows(logits, labels, tp.group, write_grad=True)
        count = (labels >= 0).sum().to(rows.dtype)
        loss = rows.sum() / count.clamp_min(1.0)
        ctx.tp, ctx.eps, ctx.params, ctx.fused = tp, eps, (w_norm, w_lm), fused
        ctx.hshape = h.shape
        ctx.save_for_backward(h2, rstd, xg, logits, count)
        return loss

    @staticmethod
    def backward(ctx, g):
        h2, rstd, xg, dlogits, count = ctx.saved_tensors
        w_norm, w_lm = ctx.params
        alpha = (g.to(torch.float32) / count.clamp_min(1.0).to(torch.float32)).reshape(1)
        if not dlogits.is_cuda:
            alpha = alpha.to(dlogits.dtype) if dlogits.dtype == torch.float64 else alpha
        if ctx.fused:
            dxn = CG.gemm_reduce_scatter(ctx.tp.workspace, dlogits, w_lm.detach(), b_mn=True,
                                         alpha_t=alpha)
        else:
            dxg = F.linear_dgrad(dlogits, w_lm.detach(), alpha_t=alpha)
            dxn = ctx.tp.reduce_in_grad(dxg)
        F.linear_wgrad(dlogits, xg, main_grad_of(w_lm), alpha_t=alpha)
        dh = F.rmsnorm_bwd(h2, w_norm.detach(), dxn, rstd, main_grad_of(w_norm))
        return dh.view(ctx.hshape), None, None, None, None, None
