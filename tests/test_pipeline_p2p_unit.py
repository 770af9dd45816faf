"""Pipeline P2P transport with ``batch_isend_irecv`` recorded (no process group).

Counterpart of the reference's P2P unit tests (tests/unit/test_pipeline_p2p.py:59-543):
activations travel on the pipeline group and gradients on the second transport channel,
every point-to-point op is a batched launch (an unbatched send/recv would make torch
create a fresh two-rank communicator lazily), sends stay in flight until drained, and
with dynamic shapes each payload is preceded by a versioned int64 shape header that the
receiver validates before allocating the payload.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from nano_megatron_b200.parallel.group_plan import GroupKey
from nano_megatron_b200.pipeline_parallel import p2p as p2p_mod


class _Work:
    def __init__(self):
        self.waited = 0

    def wait(self):
        self.waited += 1


def _comm(monkeypatch, dynamic, header_for_recv=None):
    pp_pg, ch_pg = object(), object()
    pp = SimpleNamespace(size=4, rank=1, ranks=[10, 11, 12, 13], process_group=pp_pg)
    ch = SimpleNamespace(size=4, rank=1, ranks=[10, 11, 12, 13], process_group=ch_pg)

    def group(key):
        if key == GroupKey.PP_TRANSPORT_1:
            return ch
        raise KeyError(key)

    parallel = SimpleNamespace(pp=pp, group=group)
    calls = []

    def batch(ops):
        works = []
        for op in ops:
            kind = "send" if op.op in (torch.distributed.isend,) else "recv"
            if kind == "recv" and op.tensor.dtype == torch.int64 and header_for_recv is not None:
                op.tensor.copy_(header_for_recv)
            calls.append((kind, op.peer, "pp" if op.group is pp_pg else "grad",
                          tuple(op.tensor.shape), op.tensor.dtype))
            works.append(_Work())
        return works

    class _Op:                      # records the op without resolving group ranks
        def __init__(self, op, tensor, peer, group=None):
            self.op, self.tensor, self.peer, self.group = op, tensor, peer, group

    monkeypatch.setattr(p2p_mod.dist, "batch_isend_irecv", batch)
    monkeypatch.setattr(p2p_mod.dist, "P2POp", _Op)
    c = p2p_mod.P2PCommunicator(parallel, dtype=torch.bfloat16, device=torch.device("cpu"),
                                dynamic_shapes=dynamic)
    return c, calls


def test_static_shapes_use_one_batched_op_per_transfer_on_the_right_channel(monkeypatch):
    c, calls = _comm(monkeypatch, dynamic=False)
    act = torch.zeros(3, 2, 8, dtype=torch.bfloat16)
    c.send_activation(act, 2)                              # pp index 2 -> global rank 12
    work, buf = c.post_recv_activation((3, 2, 8), 0)       # from global rank 10
    c.send_grad(act, 0)
    gwork, gbuf = c.post_recv_grad((3, 2, 8), 2)
    assert calls == [("send", 12, "pp", (3, 2, 8), torch.bfloat16),
                     ("recv", 10, "pp", (3, 2, 8), torch.bfloat16),
                     ("send", 10, "grad", (3, 2, 8), torch.bfloat16),
                     ("recv", 12, "grad", (3, 2, 8), torch.bfloat16)]
    assert buf.shape == (3, 2, 8) and buf.dtype == torch.bfloat16 and gbuf.shape == (3, 2, 8)
    assert len(c._sends) == 2                              # both sends still in flight
    c.drain_sends(keep=1)
    assert len(c._sends) == 1
    c.drain_sends()
    assert not c._sends


def test_dynamic_shapes_send_a_validated_header_first(monkeypatch):
    hdr = torch.tensor(p2p_mod.encode_header(p2p_mod.KIND_ACTIVATION, 3, 1, (5, 2, 8)))
    c, calls = _comm(monkeypatch, dynamic=True, header_for_recv=hdr)
    c.send_activation(torch.ones(5, 2, 8, dtype=torch.bfloat16), 2, microbatch=3, chunk=1)
    assert calls[0][:3] == ("send", 12, "pp") and calls[0][3:] == ((p2p_mod.HEADER_LEN,),
                                                                    torch.int64)
    assert calls[1] == ("send", 12, "pp", (5, 2, 8), torch.bfloat16)
    sent_header = c._sends[0][1]
    # version, kind, microbatch, consumer chunk, ndim, dims, unused dims -1
    assert sent_header.tolist() == [p2p_mod.HEADER_VERSION, p2p_mod.KIND_ACTIVATION, 3, 1, 3,
                                    5, 2, 8] + [-1] * (p2p_mod.MAX_DIMS - 3)
    work, buf = c.post_recv_activation((99, 99, 99), 0, microbatch=3, chunk=1)
    assert buf.shape == (5, 2, 8)                           # the header decides the shape
    assert calls[2][0] == "recv" and calls[2][4] == torch.int64 and calls[3][3] == (5, 2, 8)
    bad = hdr.clone()
    bad[0] = p2p_mod.HEADER_VERSION + 1
    c2, _ = _comm(monkeypatch, dynamic=True, header_for_recv=bad)
    with pytest.raises(RuntimeError, match="header version"):
        c2.post_recv_activation((5, 2, 8), 0, microbatch=3, chunk=1)


@pytest.mark.parametrize("expect", [(p2p_mod.KIND_GRAD, 3, 1),       # wrong kind
                                    (p2p_mod.KIND_ACTIVATION, 4, 1),  # wrong microbatch
                                    (p2p_mod.KIND_ACTIVATION, 3, 0)])  # wrong chunk
def test_misrouted_transfer_is_rejected(monkeypatch, expect):
    hdr = torch.tensor(p2p_mod.encode_header(p2p_mod.KIND_ACTIVATION, 3, 1, (5, 2, 8)))
    c, _ = _comm(monkeypatch, dynamic=True, header_for_recv=hdr)
    kind, mb, chunk = expect
    post = c.post_recv_grad if kind == p2p_mod.KIND_GRAD else c.post_recv_activation
    with pytest.raises(RuntimeError, match="out of order"):
        post((5, 2, 8), 0, microbatch=mb, chunk=chunk)


def test_malformed_header_shape_is_rejected():
    vals = p2p_mod.encode_header(p2p_mod.KIND_GRAD, 0, 0, (4, 4))
    vals[7] = 9                       # a dim past ndim that is not -1
    with pytest.raises(RuntimeError, match="malformed"):
        p2p_mod.decode_header(vals, (p2p_mod.KIND_GRAD, 0, 0))
    with pytest.raises(ValueError):
        p2p_mod.encode_header(p2p_mod.KIND_GRAD, 0, 0, tuple(range(1, 10)))
