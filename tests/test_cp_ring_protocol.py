"""Model check of the context-parallel peer ring's signalling (pure Python, CPU).

``PeerRingContextParallelAttention`` (``context_parallel/attention.py``) keeps one K/V
slot per layer on every CP rank and, per layer and microbatch:

* forward: publish this rank's K/V into its slot, signal KV (the epoch counts publishes);
  at ring step s the attention kernel's pull warp waits until the owner's KV flag has
  reached this rank's epoch, then copies the owner's slot (owner = rank - s);
* backward (layers in reverse): the same pulls, then the fp32 dK/dV partial for every
  owner whose keys this rank's queries see is stored into the owner's return slot
  (double-buffered by the DKV epoch's parity); signal DKV; ``cp_reduce`` waits until
  EVERY rank's DKV flag has reached this rank's epoch, then adds the partials of the
  ranks whose queries see its keys (``csrc/cp_comm.cu``).

No barrier separates microbatches. The all-ranks wait of ``cp_reduce`` makes each
layer's backward a barrier: no rank starts layer l - 1's pushes (which reuse the parity
of layer l + 1) before every rank has taken layer l's partials, and no owner republishes
a slot (next microbatch's forward) before every rank has finished its backward pulls. A
random scheduler interleaves the ranks' events under these waits over several layers and
microbatches. Invariants: every pull whose keys are used reads the same microbatch's
K/V; every partial taken is the same layer and microbatch's; every run completes. Pulls
whose keys the causal layout masks out may see newer data (the kernel never uses them).
Two weaker variants must be caught: waiting only for the ranks whose partials are taken
(in the contiguous causal layout the last rank then runs two layers ahead and overwrites
a return slot before its owner took it), and not waiting at all.
"""

from __future__ import annotations

import random

import pytest


class ProtocolRace(AssertionError):
    pass


def _sees(layout: str, n: int):
    if layout == "contiguous":           # causal: rank u's queries see keys of ranks <= u
        return lambda u, r: r <= u
    return lambda u, r: True             # zig-zag: every rank holds early and late chunks


def _program(r, n, layers, micro, sees, wait):
    prog = []
    for m in range(micro):
        for l in range(layers):
            prog.append(("publish", l, m))
            prog.append(("sig_kv",))
            for s in range(1, n):
                prog.append(("pull", l, m, (r - s) % n))
        for l in reversed(range(layers)):
            for s in range(1, n):
                src = (r - s) % n
                prog.append(("pull", l, m, src))
                if sees(r, src):
                    prog.append(("push", l, m, src))
            prog.append(("sig_dkv",))
            if wait == "all":
                prog.append(("wait_all",))
            for u in range(n):
                if u != r and sees(u, r):
                    prog.append(("take", l, m, u, wait == "mask"))
    return prog


def simulate(n, layers, micro, layout, seed, wait="all") -> None:
    rng = random.Random(seed)
    sees = _sees(layout, n)
    progs = [_program(r, n, layers, micro, sees, wait) for r in range(n)]
    pc = [0] * n
    kv_epoch = [0] * n
    dkv_epoch = [0] * n
    flag_kv = [[0] * n for _ in range(n)]        # [reader][writer]
    flag_dkv = [[0] * n for _ in range(n)]
    slot = [[None] * layers for _ in range(n)]    # [owner][layer] -> microbatch
    ret = [[[None] * n for _ in range(2)] for _ in range(n)]   # [owner][parity][src]

    def ready(r, ev):
        if ev[0] == "pull":
            return flag_kv[r][ev[3]] >= kv_epoch[r]
        if ev[0] == "take":
            return (not ev[4]) or flag_dkv[r][ev[3]] >= dkv_epoch[r]
        if ev[0] == "wait_all":
            return all(flag_dkv[r][u] >= dkv_epoch[r] for u in range(n))
        return True

    def run(r, ev):
        kind = ev[0]
        if kind == "publish":
            slot[r][ev[1]] = ev[2]
        elif kind == "sig_kv":
            kv_epoch[r] += 1
            for d in range(n):
                flag_kv[d][r] = kv_epoch[r]
        elif kind == "pull":
            _, l, m, src = ev
            if sees(r, src) and slot[src][l] != m:
                raise ProtocolRace(f"rank {r} pulled layer {l} of rank {src} for microbatch "
                                   f"{m} and got microbatch {slot[src][l]}")
        elif kind == "push":
            _, l, m, owner = ev
            ret[owner][(dkv_epoch[r] + 1) & 1][r] = (l, m)
        elif kind == "sig_dkv":
            dkv_epoch[r] += 1
            for d in range(n):
                flag_dkv[d][r] = dkv_epoch[r]
        elif kind == "take":
            _, l, m, u, _w = ev
            got = ret[r][dkv_epoch[r] & 1][u]
            if got != (l, m):
                raise ProtocolRace(f"rank {r} took {got} from rank {u} for layer {l}, "
                                   f"microbatch {m}")

    while True:
        cands = [r for r in range(n) if pc[r] < len(progs[r]) and ready(r, progs[r][pc[r]])]
        if not cands:
            if all(pc[r] == len(progs[r]) for r in range(n)):
                return
            raise ProtocolRace("deadlock")
        r = rng.choice(cands)
        run(r, progs[r][pc[r]])
        pc[r] += 1


@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
@pytest.mark.parametrize("n", [2, 3, 4])
def test_peer_ring_protocol_is_race_free(n, layout):
    for seed in range(200):
        simulate(n, layers=3, micro=3, layout=layout, seed=seed)


def test_waiting_only_for_the_contributing_ranks_is_caught():
    with pytest.raises(ProtocolRace):
        for seed in range(400):
            simulate(3, layers=3, micro=2, layout="contiguous", seed=seed, wait="mask")


@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_not_waiting_is_caught(layout):
    with pytest.raises(ProtocolRace):
        for seed in range(400):
            simulate(2, layers=2, micro=3, layout=layout, seed=seed, wait="none")
