"""Pipeline point-to-point transport over NCCL (gloo on CPU).

Activations (forward direction) and activation gradients (backward direction)
travel on two different communicators of the same PP ranks (the PP group and
the PP_TRANSPORT_1 channel). Each direction is then an in-order message stream
between neighbours, so a rank that blocks on a receive can never hold up a
send the peer needs first: no deadlock regardless of how the schedule
interleaves F and B (the reference colours sources over three communicators for
the same purpose, src/nano_megatron/pipeline_parallel/p2p.py:84-149).

Sends are asynchronous; the tensor is kept alive until the send completes.
Receives can be posted early (``post_recv``) and waited on right before the
compute that needs them, so transfers overlap compute (``overlap_p2p``).
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
    def _isend(self, t: torch.Tensor, dst: int, group) -> None:
        t = t.contiguous()
        if self.dynamic:
            hdr = torch.zeros(HEADER_LEN, dtype=torch.int64, device=t.device)
            hdr[0], hdr[1] = HEADER_VERSION, t.ndim
            hdr[2:2 + t.ndim] = torch.tensor(t.shape, dtype=torch.int64)
            self._sends.append((dist.isend(hdr, dst, group=group.process_group), hdr))
        self._sends.append((dist.isend(t, dst, group=group.process_group), t))

    def _irecv(self, shape, src: int, group):
        if self.dynamic:
            hdr = torch.empty(HEADER_LEN, dtype=torch.int64, device=self.device)
            dist.recv(hdr, src, group=group.process_group)
            if int(hdr[0]) != HEADER_VERSION:
                raise RuntimeError("pipeline header version mismatch")
            nd = int(hdr[1])
            shape = tuple(int(x) for x in hdr[2:2 + nd].tolist())
        buf = torch.empty(shape, dtype=self.dtype, device=self.device)
        work = dist.irecv(buf, src, group=group.process_group)
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
        """Create the communicators in a fixed order on every rank (1-element all-reduce)."""
        for g in (self.pp, self.grad_group):
            if g.size > 1 and g.process_group is not None:
                t = torch.zeros(1, device=self.device)
                dist.all_reduce(t, group=g.process_group)
