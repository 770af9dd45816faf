"""Model check of the fused collectives' signalling protocol (pure Python, CPU).

Each TP rank runs the same sequence of collectives on one stream, in the order the
kernels implement (``nano_megatron_b200/ops/comm_gemm.py``, ``csrc/comm_ops.cu``):

* AG call: publish own shard into slot[parity(e + 1)] -> signal (e += 1, flag[dst][src] =
  e for every dst) -> GEMM, which for every owner waits flag[me][owner] >= e and then
  reads owner's slot[parity(e)]; each such read is a separate event that may happen at
  any later point while the GEMM runs;
* RS call: GEMM stores this rank's partial into staging[owner][parity(e + 1)][me] for
  every owner (separate events) -> signal -> reduce: waits flag[me][src] >= e for all
  src, then reads staging[me][parity(e)][src] (separate events).

A random scheduler interleaves the ranks' events (a stream executes its events in
order, a kernel's per-peer reads in any order) while honouring the waits. Invariants:
every read returns the data of the same call, and every run completes (no deadlock).
The single-buffer variant (no parity alternation) must be caught racing, which shows the
checker can find the bug class it guards against.
"""

from __future__ import annotations

import random

import pytest


class ProtocolRace(AssertionError):
    pass


def _program(rank: int, size: int, calls: list[str], double_buffer: bool) -> list:
    """Per-rank event list. Events: ("ag_pub", k) ("sig", ch) ("ag_read", k, owner)
    ("rs_write", k, owner) ("rs_read", k, src)."""
    ev = []
    for k, kind in enumerate(calls):
        if kind == "AG":
            ev.append(("ag_pub", k))
            ev.append(("sig", "AG"))
            for o in range(size):
                ev.append(("ag_read", k, o))
        else:
            for o in range(size):
                ev.append(("rs_write", k, o))
            ev.append(("sig", "RS"))
            for s in range(size):
                ev.append(("rs_read", k, s))
    return ev


def simulate(size: int, calls: list[str], seed: int, double_buffer: bool = True) -> None:
    rng = random.Random(seed)
    par = (lambda e: e & 1) if double_buffer else (lambda e: 0)
    progs = [_program(r, size, calls, double_buffer) for r in range(size)]
    pc = [0] * size
    epoch = [{"AG": 0, "RS": 0} for _ in range(size)]
    flags = [{"AG": [0] * size, "RS": [0] * size} for _ in range(size)]
    ag_slot = [[None, None] for _ in range(size)]                    # [rank][parity]
    rs_stage = [[[None] * size for _ in range(2)] for _ in range(size)]  # [owner][par][src]
    call_epoch = [dict() for _ in range(size)]     # (rank, k) -> epoch seen by that call

    def ready(r):
        e = progs[r][pc[r]]
        if e[0] == "ag_read":
            k, o = e[1], e[2]
            return flags[r]["AG"][o] >= call_epoch[r][("AG", k)]
        if e[0] == "rs_read":
            k, s = e[1], e[2]
            return flags[r]["RS"][s] >= call_epoch[r][("RS", k)]
        return True

    def candidates():
        out = []
        for r in range(size):
            if pc[r] >= len(progs[r]):
                continue
            # a kernel's per-peer reads/writes may run in any order: expose every event of
            # the current read/write group, not just the first
            i = pc[r]
            kind = progs[r][i][0]
            j = i
            while j < len(progs[r]) and progs[r][j][0] == kind and kind.endswith(
                    ("_read", "_write")) and progs[r][j][1] == progs[r][i][1]:
                j += 1
            group = range(i, max(j, i + 1))
            for g in group:
                out.append((r, g))
        return out

    steps = 0
    while any(pc[r] < len(progs[r]) for r in range(size)):
        steps += 1
        if steps > 100000:
            raise AssertionError("simulation did not terminate")
        opts = []
        for r, g in candidates():
            saved = pc[r]
            pc[r] = g
            ok = ready(r)
            pc[r] = saved
            if ok:
                opts.append((r, g))
        if not opts:
            raise AssertionError(f"deadlock at pcs {pc}")
        r, g = rng.choice(opts)
        # move the chosen event to the front of its group, then execute it
        progs[r][pc[r]], progs[r][g] = progs[r][g], progs[r][pc[r]]
        e = progs[r][pc[r]]
        pc[r] += 1
        if e[0] == "ag_pub":
            k = e[1]
            ag_slot[r][par(epoch[r]["AG"] + 1)] = ("x", r, k)
            call_epoch[r][("AG", k)] = epoch[r]["AG"] + 1
        elif e[0] == "sig":
            ch = e[1]
            epoch[r][ch] += 1
            for d in range(size):
                flags[d][ch][r] = epoch[r][ch]
        elif e[0] == "ag_read":
            k, o = e[1], e[2]
            got = ag_slot[o][par(call_epoch[r][("AG", k)])]
            if got != ("x", o, k):
                raise ProtocolRace(f"rank {r} call {k} read {got} from owner {o}")
        elif e[0] == "rs_write":
            k, o = e[1], e[2]
            e_next = epoch[r]["RS"] + 1
            call_epoch[r][("RS", k)] = e_next
            rs_stage[o][par(e_next)][r] = ("p", r, k)
        elif e[0] == "rs_read":
            k, s = e[1], e[2]
            got = rs_stage[r][par(call_epoch[r][("RS", k)])][s]
            if got != ("p", s, k):
                raise ProtocolRace(f"rank {r} call {k} reduced {got} from {s}")


CALL_MIXES = [["AG"] * 6, ["RS"] * 6, ["AG", "RS"] * 4, ["AG", "AG", "RS", "AG", "RS", "RS"]]


@pytest.mark.parametrize("size", [2, 3, 4])
@pytest.mark.parametrize("mix", range(len(CALL_MIXES)))
def test_double_buffered_protocol_is_race_free(size, mix):
    for seed in range(150):
        simulate(size, CALL_MIXES[mix], seed)


def test_single_buffer_variant_is_caught():
    found = 0
    for seed in range(300):
        try:
            simulate(3, ["AG"] * 6, seed, double_buffer=False)
        except ProtocolRace:
            found += 1
    assert found > 0
