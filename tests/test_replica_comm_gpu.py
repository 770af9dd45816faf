"""Fused data-parallel reduction + sharded AdamW + parameter all-gather (csrc/dp_comm.cu)
against fp32 PyTorch references.

The replicas are emulated inside one process on one GPU: every "peer" heap is local
memory and the ranks' kernels are issued phase by phase (all signals, then all
reductions, then all updates, then all signals, then all waits), so no kernel waits on a
flag set by a kernel launched after it. The two-GPU path through the strategies is in
``test_replica_multigpu.py``.
"""

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.data_parallel.replica_comm import CH_GRAD, CH_PARAM, ReplicaComm  # noqa: E402
from nano_megatron_b200.distributed.symmetric import SymmetricHeap  # noqa: E402
from nano_megatron_b200.ops._ext import status_word  # noqa: E402

DEV = torch.device("cuda")


def _bucket(index, offset, numel, rank, world, slices):
    shard = -(-numel // world)
    return SimpleNamespace(index=index, offset=offset, numel=numel, rank=rank,
                           shard_numel=shard, padded_numel=shard * world,
                           slices=[SimpleNamespace(start=a, end=e, counted=c)
                                   for a, e, c in slices])


def _adamw_ref(p, g, m, v, *, lr, b1, b2, eps, wd, step, gs):
    g = g * gs
    p = p * (1 - lr * wd)
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    p = p - (lr / bc1) * m / (v.sqrt() / bc2 ** 0.5 + eps)
    return p, m, v


@pytest.mark.parametrize("world", [2, 4])
def test_reduce_update_gather_matches_fp32(world):
    torch.manual_seed(world)
    # bucket 0: 1001 elements (shards start off a 4-element boundary: scalar path);
    # bucket 1: 8192 elements at an aligned offset (vector path); one slice not counted
    layout = [(0, 1001, [(0, 600, True), (600, 1001, False)]),
              (1008, 8192, [(0, 5000, True), (5000, 8192, True)])]
    total = 1008 + 8192
    heaps = SymmetricHeap.emulated(world, ReplicaComm.regions(total, torch.bfloat16,
                                                              torch.float32), DEV)
    comms = [ReplicaComm(h, group=None) for h in heaps]
    buckets = [[_bucket(i, off, n, r, world, sl) for i, (off, n, sl) in enumerate(layout)]
               for r in range(world)]
    grads = [c.flat_tensors(total, torch.bfloat16, torch.float32)[1] for c in comms]
    params = [c.flat_tensors(total, torch.bfloat16, torch.float32)[0] for c in comms]
    for r in range(world):
        grads[r].copy_(torch.randn(total, device=DEV))
        comms[r].prepare(SimpleNamespace(buckets=buckets[r], device=DEV), lambda s: s.counted)
    orig = torch.stack([g.clone() for g in grads])
    full = orig.sum(0)
    state = {}
    for r in range(world):
        for b in buckets[r]:
            n = b.shard_numel
            state[(r, b.index)] = [torch.randn(n, device=DEV), torch.randn(n, device=DEV) * 0.1,
                                   torch.rand(n, device=DEV) * 0.01]
    hp = dict(lr=1e-2, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, step=3)
    gs = torch.tensor([0.37], device=DEV)
    lr_t = torch.tensor([hp["lr"]], device=DEV)
    ref_state = {k: [t.clone() for t in v] for k, v in state.items()}

    for c in comms:
        c.signal(CH_GRAD)
    partials = {}
    for r, c in enumerate(comms):
        for b in buckets[r]:
            partials[(r, b.index)] = c.reduce(b, lambda x: x.offset).clone()
    for r, c in enumerate(comms):
        for b in buckets[r]:
            m, ea, es = state[(r, b.index)]
            c.adamw_gather(b, lambda x: x.offset, m, ea, es, lr=hp["lr"], betas=(hp["b1"], hp["b2"]),
                           eps=hp["eps"], wd=hp["wd"], step=hp["step"], grad_scale=gs, lr_t=lr_t)
    for c in comms:
        c.signal(CH_PARAM)
    for c in comms:
        c.wait(CH_PARAM)
    torch.cuda.synchronize()
    assert int(status_word(DEV).item()) == 0

    for r in range(world):
        for b in buckets[r]:
            lo = b.rank * b.shard_numel
            hi = min(lo + b.shard_numel, b.numel)
            if hi <= lo:
                continue
            a, e = b.offset + lo, b.offset + hi
            # the shard holds the replica sum (in place)
            torch.testing.assert_close(grads[r][a:e], full[a:e], rtol=1e-6, atol=1e-5)
            # partial squared norms: the counted slices of this shard only
            want = sum(float((full[b.offset + max(s.start, lo):b.offset + min(s.end, hi)]
                              .double() ** 2).sum())
                       for s in b.slices if s.counted and min(s.end, hi) > max(s.start, lo))
            got = float(partials[(r, b.index)].double().sum())
            assert abs(got - want) <= 1e-4 * max(1.0, want), (r, b.index, got, want)
            # AdamW on the shard, bf16 result in EVERY rank's parameter buffer
            p0, m0, v0 = ref_state[(r, b.index)]
            n = hi - lo
            p1, m1, v1 = _adamw_ref(p0[:n], full[a:e], m0[:n], v0[:n], lr=hp["lr"], b1=hp["b1"],
                                    b2=hp["b2"], eps=hp["eps"], wd=hp["wd"], step=hp["step"],
                                    gs=0.37)
            got_p, got_m, got_v = state[(r, b.index)]
            torch.testing.assert_close(got_p[:n], p1, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(got_m[:n], m1, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(got_v[:n], v1, rtol=1e-5, atol=1e-7)
            for q in range(world):
                assert torch.equal(params[q][a:e], got_p[:n].to(torch.bfloat16)), (r, q, b.index)


def test_replica_wait_times_out_with_status():
    """A replica that never signals: the bounded wait gives up (~1 s), records 0x401 and
    returns; the context stays usable."""
    heaps = SymmetricHeap.emulated(2, ReplicaComm.regions(64, torch.bfloat16, torch.float32),
                                   DEV)
    comm = ReplicaComm(heaps[0], group=None)
    comm.signal(CH_PARAM)              # replica 1 never signals this epoch
    comm.wait(CH_PARAM)
    torch.cuda.synchronize()
    st = status_word(DEV)
    assert int(st.item()) == 0x401
    st.zero_()
    y = torch.randn(64, 64, device=DEV) @ torch.randn(64, 64, device=DEV)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
