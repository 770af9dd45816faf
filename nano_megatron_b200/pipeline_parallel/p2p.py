"""Pipeline point-to-point transport over NCCL (gloo on CPU).

Activations (forward direction) and activation gradients (backward direction)
travel on two different communicators of the same PP ranks (the PP group and
the PP_TRANSPORT_1 channel). Each direction is then an in-order message stream
between neighbours, so a rank that blocks on a receive can never hold up a
send the peer needs first: no deadlock regardless of how the schedule
interleaves F and B (the reference colours sources over three communicators for
the same purpose, src/nano_megatron/pipeline_parallel/p2p.py:84-149).

Sends are asynchronous; the tensor is kept alive until the send completes, and
the executor decides how many stay in flight (``overlap_p2p``). Receives are
posted by the executor right before the action that consumes them.
Shapes are static (``[S_local(/TP), B, H]``) or, with dynamic shapes, each
payload is preceded by an int64 header carrying (version, ndim, dims...).
"""

from __future__ import annotations

from collections import deque

import torch
import torch.distributed as dist

from nano_megatron_b200.parallel.group_plan import GroupKey

HEADER_VERSION = 1
HEADER_LEN = 10


class P2PCommunicator:
    def __init__(self, parallel, *, dtype: torch.dtype, device: torch.device,
                 dynamic_shapes: bool = False) -> None:
        self.parallel = parallel
        self.pp = parallel.pp
        try:
            self.grad_group = parallel.group(GroupKey.PP_TRANSPORT_1)
        except KeyError:
            self.grad_group = self.pp
        self.dtype = dtype
        self.device = device
        self.dynamic = dynamic_shapes
        self._sends: deque = deque()

    # ranks ------------------------------------------------------------------
    def rank_at(self, pp_index: int) -> int:
        return self.pp.ranks[pp_index % self.pp.size]

    # primitives -------------------------------------------------------------
    # Every point-to-point op goes through batch_isend_irecv: batched P2P runs on the
    # group's (already initialised) communicator, whereas an unbatched send/recv makes
    # torch create a fresh 2-rank communicator lazily -- and creating one while a
    # pre-posted receive kernel spins on the peer's GPU deadlocks both ranks.
    @staticmethod
    def _op(fn, t: torch.Tensor, peer: int, group):
        return dist.batch_isend_irecv([dist.P2POp(fn, t, peer, group=group.process_group)])[0]

    def _isend(self, t: torch.Tensor, dst: int, group) -> None:
        t = t.contiguous()
        if self.dynamic:
            hdr = torch.zeros(HEADER_LEN, dtype=torch.int64, device=t.device)
            hdr[0], hdr[1] = HEADER_VERSION, t.ndim
            hdr[2:2 + t.ndim] = torch.tensor(t.shape, dtype=torch.int64)
            self._sends.append((self._op(dist.isend, hdr, dst, group), hdr))
        self._sends.append((self._op(dist.isend, t, dst, group), t))

    def _irecv(self, shape, src: int, group):
        if self.dynamic:
            hdr = torch.empty(HEADER_LEN, dtype=torch.int64, device=self.device)
            self._op(dist.irecv, hdr, src, group).wait()
            if int(hdr[0]) != HEADER_VERSION:
                raise RuntimeError("pipeline header version mismatch")
            nd = int(hdr[1])
            shape = tuple(int(x) for x in hdr[2:2 + nd].tolist())
        buf = torch.empty(shape, dtype=self.dtype, device=self.device)
        work = self._op(dist.irecv, buf, src, group)
        return work, buf

    def send_activation(self, t: torch.Tensor, dst_pp: int) -> None:
        self._isend(t.detach(), self.rank_at(dst_pp), self.pp)

    def post_recv_activation(self, shape, src_pp: int):
        return self._irecv(shape, self.rank_at(src_pp), self.pp)

    def send_grad(self, t: torch.Tensor, dst_pp: int) -> None:
        self._isend(t, self.rank_at(dst_pp), self.grad_group)

    def post_recv_grad(self, shape, src_pp: int):
        return self._irecv(shape, self.rank_at(src_pp), self.grad_group)

    def drain_sends(self, keep: int = 0) -> None:
        while len(self._sends) > keep:
            work, _ = self._sends.popleft()
            work.wait()

    def warmup(self) -> None:
        """Initialise every multi-rank communicator this rank uses, in one fixed order on
        all ranks, before the first pipeline transfer (a 1-element all-reduce each): the
        TP/CP/EP/DP/replica groups first, then the two pipeline channels. No lazy
        communicator creation can then happen while a receive is outstanding."""
        from nano_megatron_b200.parallel.group_plan import GroupKey

        keys = (GroupKey.TP, GroupKey.CP, GroupKey.EP, GroupKey.DP_AXIS, GroupKey.TP_CP,
                GroupKey.TP_EP, GroupKey.DENSE_REPLICA, GroupKey.EXPERT_REPLICA,
                GroupKey.BATCH_REPLICA, GroupKey.EMBEDDING)
        groups = []
        for k in keys:
            try:
                groups.append(self.parallel.group(k))
            except KeyError:
                continue
        groups += [self.pp, self.grad_group]
        seen = set()
        for g in groups:
            pg = g.process_group
            if g.size > 1 and pg is not None and id(pg) not in seen:
                seen.add(id(pg))
                t = torch.zeros(1, device=self.device)
                dist.all_reduce(t, group=pg)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
