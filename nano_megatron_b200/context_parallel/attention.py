"""Context-parallel attention cores (all-gather and ring)."""

from __future__ import annotations

from typing import Protocol

import torch
import torch.distributed as dist

from nano_megatron_b200.ops import functional as F
from nano_megatron_b200.tensor_parallel.comm import all_gather_dim0, reduce_scatter_dim0

from .utils import chunk_ids, gathered_to_global_order, local_positions


class ContextParallelAttention(Protocol):
    """What the fused attention block (``models/gpt/blocks.py``) calls on its attention
    core: the local core and every context-parallel core implement it.

    ``forward`` writes the output of this rank's query rows into ``o`` ([S, B, Hq, D]
    view) and returns the base-2 log-sum-exp [B, Hq, S]; ``backward`` writes dq, dk, dv.
    q/k/v are [B, S, H, D] strided views of the fused QKV buffer; ``mb`` carries the
    microbatch's positions and layer. ``applies_inverse_rope``: whether ``backward``
    already returns gradients with respect to the pre-rotation q/k (else the block
    applies the inverse rotation). The reference's interface of the same name takes and
    returns [B, H, S, D] tensors (src/nano_megatron/context_parallel/interface.py:10-22);
    that form is :func:`nano_megatron_b200.nn.kernels.B200KernelBackend.local_attention`.
    """

    applies_inverse_rope: bool

    def forward(self, q, k, v, o, mb) -> torch.Tensor: ...

    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq) -> None: ...


class _CPBase:
    """Shared chunk bookkeeping; inverse RoPE is applied by the attention block."""

    applies_inverse_rope = False

    def __init__(self, group, *, load_balance: bool = False) -> None:
        self.group = group
        self.load_balance = load_balance

    def local_positions(self, seq_local: int, rank: int, size: int) -> torch.Tensor:
        return local_positions(seq_local, rank, size, self.load_balance)

    def q_chunks(self, seq_local: int, rank: int | None = None):
        """(row start, rows, absolute position offset) of each query chunk of ``rank``
        (default: this rank)."""
        size = self.group.size
        rank = self.group.rank if rank is None else rank
        if not self.load_balance:
            return [(0, seq_local, rank * seq_local)]
        c = seq_local // 2
        a, b = chunk_ids(rank, size, True)
        return [(0, c, a * c), (c, c, b * c)]


def _kv_rows(q, k, v):
    """The [S, B, 2*Hkv*D] strided row view holding k|v (adjacent in the QKV buffer)."""
    B, S, hkv, D = k.shape
    base = k.transpose(0, 1)  # [S, B, Hkv, D]
    return torch.as_strided(base, (S, B, 2 * hkv * D), (base.stride(0), base.stride(1), 1))


class AllGatherContextParallelAttention(_CPBase):
    def _gather(self, k, v):
        B, S, hkv, D = k.shape
        kv = _kv_rows(None, k, v).contiguous()                     # [S, B, 2HkvD]
        full = all_gather_dim0(kv, self.group)                     # rank-major
        size = self.group.size
        if self.load_balance:
            c = S // 2
            parts = full.view(size, 2, c, B, 2 * hkv * D)
            order = gathered_to_global_order(size, True)
            full = torch.cat([parts[r, h] for r, h in order], 0)
        kvf = full.view(size * S, B, 2, hkv, D)
        return kvf[:, :, 0].transpose(0, 1), kvf[:, :, 1].transpose(0, 1), full

    def forward(self, q, k, v, o, mb):
        kf, vf, full = self._gather(k, v)
        o_bs = o.transpose(0, 1)
        B, Sq, Hq, D = o_bs.shape
        lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32)
        for start, rows, off in self.q_chunks(Sq):
            oc, lc = F.attention_fwd(q[:, start:start + rows], kf, vf, causal=True,
                                     q_offset=off, k_offset=0)
            o_bs[:, start:start + rows].copy_(oc)
            lse[:, :, start:start + rows].copy_(lc)
        mb.extra["cp_kv_full"] = full
        return lse

    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq):
        full = mb.extra.pop("cp_kv_full", None)
        if full is None:
            kf, vf, full = self._gather(k, v)
        else:
            B, S, hkv, D = k.shape
            kvf = full.view(-1, B, 2, hkv, D)
            kf, vf = kvf[:, :, 0].transpose(0, 1), kvf[:, :, 1].transpose(0, 1)
        dfull = torch.zeros(full.shape, dtype=torch.float32, device=full.device)
        B, Stot, hkv, D = kf.shape
        dview = dfull.view(Stot, B, 2, hkv, D)
        o_bs = o.transpose(0, 1)
        for start, rows, off in self.q_chunks(q.shape[1]):
            dkc = torch.empty(B, Stot, hkv, D, device=q.device, dtype=q.dtype)
            dvc = torch.empty_like(dkc)
            F.attention_bwd(q[:, start:start + rows], kf, vf, o_bs[:, start:start + rows],
                            do[:, start:start + rows], lse[:, :, start:start + rows].contiguous(),
                            dq[:, start:start + rows], dkc, dvc, causal=True, q_offset=off,
                            k_offset=0)
            dview[:, :, 0] += dkc.transpose(0, 1).float()
            dview[:, :, 1] += dvc.transpose(0, 1).float()
        size = self.group.size
        S = k.shape[1]
        if self.load_balance:
            c = S // 2
            chunks = dfull.view(2 * size, c, B, 2 * hkv * D)
            order = gathered_to_global_order(size, True)
            ranked = torch.empty_like(dfull).view(size, 2, c, B, 2 * hkv * D)
            for g, (r, h) in enumerate(order):
                ranked[r, h] = chunks[g]
            dfull = ranked.view(size * S, B, 2 * hkv * D)
        local = reduce_scatter_dim0(dfull.view(size * S, B, 2 * hkv * D), self.group)
        lv = local.view(S, B, 2, hkv, D)
        dk.copy_(lv[:, :, 0].transpose(0, 1))
        dv.copy_(lv[:, :, 1].transpose(0, 1))


def _merge(o_acc, lse_acc, o_new, lse_new):
    """Combine two normalised partial attention outputs by their base-2 LSEs (in place)."""
    m = torch.maximum(lse_acc, lse_new)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w1 = torch.exp2(lse_acc - m_safe)
    w2 = torch.exp2(lse_new - m_safe)
    tot = w1 + w2
    scale1 = torch.where(tot > 0, w1 / tot, torch.zeros_like(tot))
    scale2 = torch.where(tot > 0, w2 / tot, torch.zeros_like(tot))
    # lse [B, H, S] -> weights [B, S, H, 1]
    o_acc.mul_(scale1.permute(0, 2, 1).unsqueeze(-1)).add_(
        o_new.float() * scale2.permute(0, 2, 1).unsqueeze(-1))
    lse_acc.copy_(torch.where(tot > 0, m_safe + torch.log2(tot), lse_acc))


class RingContextParallelAttention(_CPBase):
    """K/V rotate around the CP ring; partial outputs merged by LSE; masked blocks skipped.

    Each step starts the next K/V rotation (P2P on the communicator's stream) before
    computing on the current block and waits for it only afterwards, so the transfer
    overlaps the flash-attention blocks. In the backward pass the dK/dV partial computed
    for a source rank's K/V is sent straight back to that rank (fp32) as soon as it is
    complete, instead of travelling the ring with an accumulator; the owner adds the
    partials in step order. Fully masked (causal) source blocks send nothing. The reference
    rotates K/V with blocking exchanges and carries a 4-tensor fp32 accumulator stack once
    around the ring (src/nano_megatron/context_parallel/ring.py:82-101, 169-250).
    """

    def _ring_pairs(self, rank_src: int, Sq: int, Sk: int, rank_q: int | None = None):
        """(q start, q rows, q offset, k start, k rows, k offset) sub-blocks of rank
        ``rank_q``'s queries (default: this rank) against the keys of ``rank_src``."""
        size = self.group.size
        qs = self.q_chunks(Sq, rank_q)
        if not self.load_balance:
            ks = [(0, Sk, rank_src * Sk)]
        else:
            c = Sk // 2
            a, b = chunk_ids(rank_src, size, True)
            ks = [(0, c, a * c), (c, c, b * c)]
        out = []
        for qstart, qrows, qoff in qs:
            for kstart, krows, koff in ks:
                if koff > qoff + qrows - 1:
                    continue  # entirely above the causal diagonal
                out.append((qstart, qrows, qoff, kstart, krows, koff))
        return out

    def _exchange(self, send: torch.Tensor | None, to: int, recv: torch.Tensor | None,
                  frm: int) -> list:
        """Start a send to / receive from group-local ranks; returns the pending works."""
        g = self.group
        ops = []
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send, g.ranks[to], group=g.process_group))
        if recv is not None:
            ops.append(dist.P2POp(dist.irecv, recv, g.ranks[frm], group=g.process_group))
        return dist.batch_isend_irecv(ops) if ops else []

    def _start_rotate(self, t: torch.Tensor):
        """Send ``t`` to the next rank of the ring and receive the previous rank's block."""
        g = self.group
        recv = torch.empty_like(t)
        return recv, self._exchange(t, (g.rank + 1) % g.size, recv, (g.rank - 1) % g.size)

    @staticmethod
    def _wait(works) -> None:
        for w in works:
            w.wait()

    def forward(self, q, k, v, o, mb):
        B, Sq, Hq, D = q.shape
        hkv = k.shape[2]
        kv = _kv_rows(q, k, v).contiguous()
        o_acc = torch.zeros(B, Sq, Hq, D, device=q.device, dtype=torch.float32)
        lse_acc = torch.full((B, Hq, Sq), float("-inf"), device=q.device, dtype=torch.float32)
        g = self.group
        cur = kv
        for step in range(g.size):
            src = (g.rank - step) % g.size
            nxt, works = self._start_rotate(cur) if step + 1 < g.size else (None, [])
            view = cur.view(-1, B, 2, hkv, D)
            kb, vb = view[:, :, 0].transpose(0, 1), view[:, :, 1].transpose(0, 1)
            for qs, qr, qo, ks, kr, ko in self._ring_pairs(src, Sq, kb.shape[1]):
                on, ln = F.attention_fwd(q[:, qs:qs + qr], kb[:, ks:ks + kr], vb[:, ks:ks + kr],
                                         causal=True, q_offset=qo, k_offset=ko)
                _merge(o_acc[:, qs:qs + qr], lse_acc[:, :, qs:qs + qr], on, ln)
            self._wait(works)
            if nxt is not None:
                cur = nxt
        o.transpose(0, 1).copy_(o_acc.to(o.dtype))
        return lse_acc

    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq):
        B, Sq, Hq, D = q.shape
        hkv = k.shape[2]
        g = self.group
        kv = _kv_rows(q, k, v).contiguous()
        Sk = kv.shape[0]
        own = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)
        dq_acc = torch.zeros(B, Sq, Hq, D, dtype=torch.float32, device=q.device)
        o_bs = o.transpose(0, 1)
        cur = kv
        returns, incoming = [], []          # pending dK/dV partial exchanges
        for step in range(g.size):
            src = (g.rank - step) % g.size
            nxt, works = self._start_rotate(cur) if step + 1 < g.size else (None, [])
            view = cur.view(-1, B, 2, hkv, D)
            kb, vb = view[:, :, 0].transpose(0, 1), view[:, :, 1].transpose(0, 1)
            pairs = self._ring_pairs(src, Sq, Sk)
            part = own if step == 0 else \
                (torch.zeros(kv.shape, dtype=torch.float32, device=q.device) if pairs else None)
            dview = part.view(-1, B, 2, hkv, D) if part is not None else None
            for qs, qr, qo, ks, kr, ko in pairs:
                dqc = torch.empty(B, qr, Hq, D, device=q.device, dtype=q.dtype)
                dkc = torch.empty(B, kr, hkv, D, device=q.device, dtype=q.dtype)
                dvc = torch.empty_like(dkc)
                F.attention_bwd(q[:, qs:qs + qr], kb[:, ks:ks + kr], vb[:, ks:ks + kr],
                                o_bs[:, qs:qs + qr], do[:, qs:qs + qr],
                                lse[:, :, qs:qs + qr].contiguous(), dqc, dkc, dvc, causal=True,
                                q_offset=qo, k_offset=ko)
                dq_acc[:, qs:qs + qr] += dqc.float()
                dview[ks:ks + kr, :, 0] += dkc.transpose(0, 1).float()
                dview[ks:ks + kr, :, 1] += dvc.transpose(0, 1).float()
            if step > 0:
                # Return this partial to the owner of the K/V just used, and receive the
                # partial that rank (rank + step) computed for this rank's K/V, if any.
                frm = (g.rank + step) % g.size
                recv = torch.empty(kv.shape, dtype=torch.float32, device=q.device) \
                    if self._ring_pairs(g.rank, Sq, Sk, rank_q=frm) else None
                returns.append((part, self._exchange(part, src, recv, frm)))
                if recv is not None:
                    incoming.append(recv)
            self._wait(works)
            if nxt is not None:
                cur = nxt
        for _part, works in returns:
            self._wait(works)
        for recv in incoming:           # step order: deterministic summation
            own += recv
        dq.copy_(dq_acc.to(dq.dtype))
        lv = own.view(-1, B, 2, hkv, D)
        dk.copy_(lv[:, :, 0].transpose(0, 1))
        dv.copy_(lv[:, :, 1].transpose(0, 1))


CH_KV, CH_DKV = 0, 1


class PeerRingContextParallelAttention(RingContextParallelAttention):
    """Ring attention whose K/V blocks travel through NVLink peer memory.

    Every rank publishes the layer's K/V block into its :class:`SymmetricHeap` slot for
    that layer (one copy, then a signal). Ring step ``i`` computes on block ``i`` with the
    flash kernels while their pull warp copies block ``i + 1`` from its owner's slot into
    a local double buffer (plain peer loads; the kernels' TMA loads then read only this
    GPU's memory). The owner is read directly, not relayed around the ring: NVSwitch gives
    every pair full bandwidth. In the backward pass the blocks are pulled again from the
    same slots, and each fp32 dK/dV partial for another rank's keys is stored into that
    rank's return slot by peer stores; after a signal the owner adds the partials of the
    ranks whose queries see its keys (the causal layout tells which) to its own. Falls back
    to the NCCL ring when no heap is attached (CPU, or a layout the heap does not cover).
    The reference rotates K/V with blocking send/receive pairs
    (src/nano_megatron/context_parallel/ring.py:82-101, 161, 247).
    """

    heap = None
    layer_slots: dict = {}
    kv_numel = 0

    def attach(self, heap, layer_slots: dict, kv_numel: int, device) -> None:
        self.heap = heap
        self.layer_slots = dict(layer_slots)
        self.kv_numel = int(kv_numel)
        self._bufs = [torch.empty(kv_numel, dtype=torch.bfloat16, device=device)
                      for _ in range(2)]
        self._dkv_numel = kv_numel

    def detach(self) -> None:
        self.heap = None
        self._bufs = []

    # ------------------------------------------------------------------ addressing
    def _slot_ptr(self, rank: int, layer: int) -> int:
        return self.heap.ptr(rank, "kv") + self.layer_slots[layer] * self.kv_numel * 2

    def _slot_view(self, layer: int) -> torch.Tensor:
        kv = self.heap.local("kv", torch.bfloat16)
        off = self.layer_slots[layer] * self.kv_numel
        return kv[off:off + self.kv_numel]

    def _ret_ptr(self, owner: int, parity: int, src: int) -> int:
        n = self.heap.size
        return self.heap.ptr(owner, "dkv") + ((parity & 1) * n + src) * self._dkv_numel * 4

    def _pull(self, src: int, layer: int, step_next: int):
        if step_next >= self.heap.size:
            return None
        h = self.heap
        return (self._slot_ptr(src, layer), self._bufs[step_next % 2],
                h.flag_slots(h.rank, CH_KV) + src * 4, h.epoch_ptr(CH_KV))

    def _usable(self, q, mb) -> bool:
        return self.heap is not None and q.is_cuda and \
            mb.extra.get("layer") in self.layer_slots

    def _block(self, step: int, own: torch.Tensor) -> torch.Tensor:
        return own if step == 0 else self._bufs[step % 2]

    # ------------------------------------------------------------------ forward
    def forward(self, q, k, v, o, mb):
        if not self._usable(q, mb):
            return super().forward(q, k, v, o, mb)
        from nano_megatron_b200.ops._ext import lib

        layer = mb.extra["layer"]
        B, Sq, Hq, D = q.shape
        hkv = k.shape[2]
        g, h = self.group, self.heap
        own = self._slot_view(layer)
        own.view(-1, B, 2 * hkv * D).copy_(_kv_rows(q, k, v))     # publish this layer's K/V
        lib().peer_signal(h.signal_targets(CH_KV), h.epoch_ptr(CH_KV))
        o_acc = torch.zeros(B, Sq, Hq, D, device=q.device, dtype=torch.float32)
        lse_acc = torch.full((B, Hq, Sq), float("-inf"), device=q.device, dtype=torch.float32)
        for step in range(g.size):
            src = (g.rank - step) % g.size
            pull = self._pull((g.rank - step - 1) % g.size, layer, step + 1)
            view = self._block(step, own).view(-1, B, 2, hkv, D)
            kb, vb = view[:, :, 0].transpose(0, 1), view[:, :, 1].transpose(0, 1)
            pairs = self._ring_pairs(src, Sq, kb.shape[1])
            if not pairs and pull is not None:
                lib().cp_pull(pull[0], pull[1], pull[2], pull[3], h.status)
            for i, (qs, qr, qo, ks, kr, ko) in enumerate(pairs):
                on, ln = F.attention_fwd(q[:, qs:qs + qr], kb[:, ks:ks + kr], vb[:, ks:ks + kr],
                                         causal=True, q_offset=qo, k_offset=ko,
                                         pull=pull if i == 0 else None)
                _merge(o_acc[:, qs:qs + qr], lse_acc[:, :, qs:qs + qr], on, ln)
        o.transpose(0, 1).copy_(o_acc.to(o.dtype))
        return lse_acc

    # ------------------------------------------------------------------ backward
    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq):
        if not self._usable(q, mb):
            return super().backward(q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq)
        from nano_megatron_b200.ops._ext import lib

        layer = mb.extra["layer"]
        B, Sq, Hq, D = q.shape
        hkv = k.shape[2]
        g, h = self.group, self.heap
        own = self._slot_view(layer)            # still this layer's K/V (published in forward)
        Sk = own.numel() // (B * 2 * hkv * D)
        mine = torch.zeros(Sk, B, 2 * hkv * D, dtype=torch.float32, device=q.device)
        dq_acc = torch.zeros(B, Sq, Hq, D, dtype=torch.float32, device=q.device)
        o_bs = o.transpose(0, 1)
        mask = 0
        for step in range(g.size):
            src = (g.rank - step) % g.size
            pull = self._pull((g.rank - step - 1) % g.size, layer, step + 1)
            view = self._block(step, own).view(-1, B, 2, hkv, D)
            kb, vb = view[:, :, 0].transpose(0, 1), view[:, :, 1].transpose(0, 1)
            pairs = self._ring_pairs(src, Sq, Sk)
            if not pairs and pull is not None:
                lib().cp_pull(pull[0], pull[1], pull[2], pull[3], h.status)
            part = mine if step == 0 else \
                (torch.zeros(Sk, B, 2 * hkv * D, dtype=torch.float32, device=q.device)
                 if pairs else None)
            dview = part.view(-1, B, 2, hkv, D) if part is not None else None
            for i, (qs, qr, qo, ks, kr, ko) in enumerate(pairs):
                dqc = torch.empty(B, qr, Hq, D, device=q.device, dtype=q.dtype)
                dkc = torch.empty(B, kr, hkv, D, device=q.device, dtype=q.dtype)
                dvc = torch.empty_like(dkc)
                F.attention_bwd(q[:, qs:qs + qr], kb[:, ks:ks + kr], vb[:, ks:ks + kr],
                                o_bs[:, qs:qs + qr], do[:, qs:qs + qr],
                                lse[:, :, qs:qs + qr].contiguous(), dqc, dkc, dvc, causal=True,
                                q_offset=qo, k_offset=ko, pull=pull if i == 0 else None)
                dq_acc[:, qs:qs + qr] += dqc.float()
                dview[ks:ks + kr, :, 0] += dkc.transpose(0, 1).float()
                dview[ks:ks + kr, :, 1] += dvc.transpose(0, 1).float()
            if step > 0 and part is not None:
                # return the partial to the owner of these keys: peer stores into its slot
                lib().cp_push(part.view(-1), self._ret_ptr(src, 0, g.rank),
                              self._ret_ptr(src, 1, g.rank), h.epoch_ptr(CH_DKV))
            # which ranks' queries see this rank's keys (they send partials back)
            frm = (g.rank + step) % g.size
            if step > 0 and self._ring_pairs(g.rank, Sq, Sk, rank_q=frm):
                mask |= 1 << frm
        lib().peer_signal(h.signal_targets(CH_DKV), h.epoch_ptr(CH_DKV))
        lib().cp_reduce(mine.view(-1), [self._ret_ptr(h.rank, 0, s) for s in range(g.size)],
                        [self._ret_ptr(h.rank, 1, s) for s in range(g.size)], mask,
                        h.flag_slots(h.rank, CH_DKV), h.epoch_ptr(CH_DKV), h.status)
        dq.copy_(dq_acc.to(dq.dtype))
        lv = mine.view(-1, B, 2, hkv, D)
        dk.copy_(lv[:, :, 0].transpose(0, 1))
        dv.copy_(lv[:, :, 1].transpose(0, 1))


class PeerAllGatherContextParallelAttention(PeerRingContextParallelAttention):
    """All-gather context parallelism whose K/V gather and dK/dV reduce-scatter go through
    NVLink peer memory instead of NCCL collectives.

    Forward: every rank publishes the layer's K/V block into its heap slot and signals;
    each peer's block is then pulled (plain peer loads after a bounded wait on the owner's
    flag) straight into its place in the global-order K/V buffer -- the zig-zag halves of
    a load-balanced layout land at their global chunk positions, so no reordering pass is
    needed -- and the flash kernels run each local query chunk against the full K/V, as
    in :class:`AllGatherContextParallelAttention`. The gathered buffer is kept for the
    backward pass. Backward: dK/dV over the full K/V are accumulated in fp32; each owner's
    rows are stored into its return slot by peer stores, and after one signal every rank
    adds the partials of all peers to its own rows (the reduce-scatter).
    Reference: src/nano_megatron/context_parallel/all_gather.py:38-113 (NCCL all-gather of
    K/V, reduce-scatter of their gradients). Falls back to the NCCL all-gather without a
    heap.
    """

    _gather = AllGatherContextParallelAttention._gather

    def _chunk_rows(self, rank: int, S: int):
        """(local row start, rows, global row start) of ``rank``'s K/V block pieces."""
        if not self.load_balance:
            return [(0, S, rank * S)]
        c = S // 2
        a, b = chunk_ids(rank, self.group.size, True)
        return [(0, c, a * c), (c, c, b * c)]

    def forward(self, q, k, v, o, mb):
        if not self._usable(q, mb):
            return AllGatherContextParallelAttention.forward(self, q, k, v, o, mb)
        from nano_megatron_b200.ops._ext import lib

        layer = mb.extra["layer"]
        B, Sq, Hq, D = q.shape
        hkv = k.shape[2]
        g, h = self.group, self.heap
        S = k.shape[1]
        row = B * 2 * hkv * D                                  # elements per sequence row
        own = self._slot_view(layer)
        own.view(-1, B, 2 * hkv * D).copy_(_kv_rows(q, k, v))  # publish this layer's K/V
        lib().peer_signal(h.signal_targets(CH_KV), h.epoch_ptr(CH_KV))
        full = torch.empty(g.size * S, B, 2 * hkv * D, device=q.device, dtype=q.dtype)
        flat = full.view(-1)
        for r in range(g.size):
            for lo, rows, glo in self._chunk_rows(r, S):
                dst = flat[glo * row:(glo + rows) * row]
                if r == g.rank:
                    dst.copy_(own[lo * row:(lo + rows) * row])
                else:
                    lib().cp_pull(self._slot_ptr(r, layer) + lo * row * 2, dst,
                                  h.flag_slots(h.rank, CH_KV) + r * 4, h.epoch_ptr(CH_KV),
                                  h.status)
        kvf = full.view(g.size * S, B, 2, hkv, D)
        kf, vf = kvf[:, :, 0].transpose(0, 1), kvf[:, :, 1].transpose(0, 1)
        o_bs = o.transpose(0, 1)
        lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32)
        for start, rows, off in self.q_chunks(Sq):
            oc, lc = F.attention_fwd(q[:, start:start + rows], kf, vf, causal=True,
                                     q_offset=off, k_offset=0)
            o_bs[:, start:start + rows].copy_(oc)
            lse[:, :, start:start + rows].copy_(lc)
        mb.extra["cp_kv_full"] = full
        return lse

    def backward(self, q, k, v, o, do, lse, dq, dk, dv, mb, inv_freq):
        if not self._usable(q, mb) or "cp_kv_full" not in mb.extra:
            return AllGatherContextParallelAttention.backward(self, q, k, v, o, do, lse, dq, dk,
                                                              dv, mb, inv_freq)
        from nano_megatron_b200.ops._ext import lib

        full = mb.extra.pop("cp_kv_full")
        B, S, hkv, D = k.shape
        Hq = q.shape[2]
        g, h = self.group, self.heap
        row = B * 2 * hkv * D
        kvf = full.view(-1, B, 2, hkv, D)
        kf, vf = kvf[:, :, 0].transpose(0, 1), kvf[:, :, 1].transpose(0, 1)
        Stot = kf.shape[1]
        dfull = torch.zeros(Stot, B, 2 * hkv * D, dtype=torch.float32, device=q.device)
        dview = dfull.view(Stot, B, 2, hkv, D)
        o_bs = o.transpose(0, 1)
        for start, rows, off in self.q_chunks(q.shape[1]):
            dkc = torch.empty(B, Stot, hkv, D, device=q.device, dtype=q.dtype)
            dvc = torch.empty_like(dkc)
            F.attention_bwd(q[:, start:start + rows], kf, vf, o_bs[:, start:start + rows],
                            do[:, start:start + rows], lse[:, :, start:start + rows].contiguous(),
                            dq[:, start:start + rows], dkc, dvc, causal=True, q_offset=off,
                            k_offset=0)
            dview[:, :, 0] += dkc.transpose(0, 1).float()
            dview[:, :, 1] += dvc.transpose(0, 1).float()
        dflat = dfull.view(-1)
        mine = torch.empty(S * row, dtype=torch.float32, device=q.device)
        for r in range(g.size):
            for lo, rows, glo in self._chunk_rows(r, S):
                part = dflat[glo * row:(glo + rows) * row]
                if r == g.rank:
                    mine[lo * row:(lo + rows) * row].copy_(part)
                else:   # peer stores into r's return slot for this source rank
                    lib().cp_push(part, self._ret_ptr(r, 0, g.rank) + lo * row * 4,
                                  self._ret_ptr(r, 1, g.rank) + lo * row * 4,
                                  h.epoch_ptr(CH_DKV))
        lib().peer_signal(h.signal_targets(CH_DKV), h.epoch_ptr(CH_DKV))
        mask = sum(1 << r for r in range(g.size) if r != g.rank)
        lib().cp_reduce(mine, [self._ret_ptr(h.rank, 0, s) for s in range(g.size)],
                        [self._ret_ptr(h.rank, 1, s) for s in range(g.size)], mask,
                        h.flag_slots(h.rank, CH_DKV), h.epoch_ptr(CH_DKV), h.status)
        lv = mine.view(S, B, 2, hkv, D)
        dk.copy_(lv[:, :, 0].transpose(0, 1))
        dv.copy_(lv[:, :, 1].transpose(0, 1))
