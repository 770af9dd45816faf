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
payload is preceded by an int64 header naming the transfer and its shape:
(version, kind, microbatch, chunk, ndim, d0..d7), unused dims -1; ``chunk`` is the
virtual stage of the *consumer*. The receiver checks the identity against the
action it is about to run and rejects a misrouted transfer (same fields as the
reference's header, src/nano_megatron/pipeline_parallel/p2p.py:279-316).
Reading a header needs its values on the host; the read waits only for the
header transfer (a side stream waits on the receive, copies the 13 values to
pinned memory and records an event the host waits on), not for the compute
queued on the current stream, so the host keeps launching ahead.
"""

from __future__ import annotations

from collections import deque

import torch
import torch.distributed as dist

from nano_megatron_b200.parallel.group_plan import GroupKey

HEADER_VERSION = 2
MAX_DIMS = 8
HEADER_LEN = 5 + MAX_DIMS
KIND_ACTIVATION, KIND_GRAD = 0, 1


def encode_header(kind: int, microbatch: int, chunk: int, shape) -> list[int]:
    shape = [int(x) for x in shape]
    if len(shape) > MAX_DIMS or any(x < 0 for x in shape):
        raise ValueError(f"pipeline tensor shape {tuple(shape)} cannot be sent (at most "
                         f"{MAX_DIMS} non-negative dims)")
    return [HEADER_VERSION, int(kind), int(microbatch), int(chunk), len(shape)] + shape + \
        [-1] * (MAX_DIMS - len(shape))


def decode_header(values, expect: tuple[int, int, int]) -> tuple[int, ...]:
    """Shape carried by a header, after checking its version and that it is the transfer
    ``expect`` = (kind, microbatch, consumer chunk)."""
    values = [int(x) for x in values]
    if len(values) != HEADER_LEN:
        raise RuntimeError(f"pipeline header has {len(values)} fields, expected {HEADER_LEN}")
    version, kind, mb, chunk, ndim = values[:5]
    if version != HEADER_VERSION:
        raise RuntimeError(f"pipeline header version {version}; this build speaks "
                           f"{HEADER_VERSION}")
    if (kind, mb, chunk) != tuple(expect):
        names = {KIND_ACTIVATION: "activation", KIND_GRAD: "gradient"}
        raise RuntimeError(
            f"pipeline transfer out of order: got {names.get(kind, kind)} of microbatch {mb} "
            f"for chunk {chunk}, this action expects {names.get(expect[0], expect[0])} of "
            f"microbatch {expect[1]} for chunk {expect[2]}")
    dims = values[5:]
    if not 0 <= ndim <= MAX_DIMS or any(d < 0 for d in dims[:ndim]) or \
            any(d != -1 for d in dims[ndim:]):
        raise RuntimeError(f"pipeline header carries a malformed shape: ndim={ndim}, "
                           f"dims={dims}")
    return tuple(dims[:ndim])


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
        self._hdr_stream = self._hdr_host = self._hdr_event = None

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

    def _isend(self, t: torch.Tensor, dst: int, group, ident) -> None:
        t = t.contiguous()
        if self.dynamic:
            hdr = torch.tensor(encode_header(*ident, t.shape), dtype=torch.int64).to(
                t.device, non_blocking=True)
            self._sends.append((self._op(dist.isend, hdr, dst, group), hdr))
        self._sends.append((self._op(dist.isend, t, dst, group), t))

    def _read_header(self, hdr: torch.Tensor, work) -> list[int]:
        if hdr.device.type != "cuda":
            work.wait()
            return hdr.tolist()
        if self._hdr_stream is None:
            self._hdr_stream = torch.cuda.Stream(hdr.device)
            self._hdr_host = torch.empty(HEADER_LEN, dtype=torch.int64, pin_memory=True)
            self._hdr_event = torch.cuda.Event()
        hs = self._hdr_stream
        hdr.record_stream(hs)
        with torch.cuda.stream(hs):
            work.wait()                        # hs (not the compute stream) waits for it
            self._hdr_host.copy_(hdr, non_blocking=True)
            self._hdr_event.record(hs)
        self._hdr_event.synchronize()
        return self._hdr_host.tolist()

    def _irecv(self, shape, src: int, group, ident):
        if self.dynamic:
            hdr = torch.empty(HEADER_LEN, dtype=torch.int64, device=self.device)
            shape = decode_header(self._read_header(hdr, self._op(dist.irecv, hdr, src, group)),
                                  ident)
        buf = torch.empty(shape, dtype=self.dtype, device=self.device)
        work = self._op(dist.irecv, buf, src, group)
        return work, buf

    # ``microbatch`` / ``chunk`` name the transfer by its consumer's action (dynamic shapes
    # carry them in the header; static shapes ignore them)
    def send_activation(self, t: torch.Tensor, dst_pp: int, microbatch: int = 0,
                        chunk: int = 0) -> None:
        self._isend(t.detach(), self.rank_at(dst_pp), self.pp,
                    (KIND_ACTIVATION, microbatch, chunk))

    def post_recv_activation(self, shape, src_pp: int, microbatch: int = 0, chunk: int = 0):
        return self._irecv(shape, self.rank_at(src_pp), self.pp,
                           (KIND_ACTIVATION, microbatch, chunk))

    def send_grad(self, t: torch.Tensor, dst_pp: int, microbatch: int = 0,
                  chunk: int = 0) -> None:
        self._isend(t, self.rank_at(dst_pp), self.grad_group, (KIND_GRAD, microbatch, chunk))

    def post_recv_grad(self, shape, src_pp: int, microbatch: int = 0, chunk: int = 0):
        return self._irecv(shape, self.rank_at(src_pp), self.grad_group,
                           (KIND_GRAD, microbatch, chunk))

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
