"""Model check of the in-kernel GEMM -> reduce-scatter's per-tile flags (pure Python, CPU).

With ``NMB_RS_IN_KERNEL=1`` the row-parallel GEMM reduces inside its epilogue
(``csrc/gemm_tcgen05.cu``, ``kEpiPeer`` with ``rs_inplace``). In call c (epoch e = c + 1)
each TP rank first computes the tiles of the rows other ranks own and stores each partial
into the owner's staging area [parity(e)][this rank], then releases that tile's flag
(= e); then it computes its own rows' tiles, and for each waits until every other rank's
flag for that tile has reached e, reads their partials and writes the sum. There is no
barrier between calls. A random scheduler interleaves the ranks' events under these waits.
Invariants: every partial read is the same call's; every run completes. Two variants must
fail: a single staging buffer (no parity) races, and own rows first deadlocks (every rank
waits for partials that nobody has written yet).
"""

from __future__ import annotations

import random

import pytest


class ProtocolFailure(AssertionError):
    pass


def _program(r, n, calls, own_rows_last):
    prog = []
    for c in range(calls):
        writes = [("write", c, o) for o in range(n) if o != r]
        reads = [("read", c, s) for s in range(n) if s != r]
        prog += (writes + reads) if own_rows_last else (reads + writes)
    return prog


def simulate(n, calls, seed, *, double_buffer=True, own_rows_last=True) -> None:
    rng = random.Random(seed)
    progs = [_program(r, n, calls, own_rows_last) for r in range(n)]
    pc = [0] * n
    flag = [[0] * n for _ in range(n)]                   # [owner][src] per-tile flag
    stage = [[[None] * n for _ in range(2)] for _ in range(n)]   # [owner][parity][src]
    par = (lambda e: e & 1) if double_buffer else (lambda e: 0)

    def ready(r, ev):
        return ev[0] != "read" or flag[r][ev[2]] >= ev[1] + 1

    while True:
        cands = [r for r in range(n) if pc[r] < len(progs[r]) and ready(r, progs[r][pc[r]])]
        if not cands:
            if all(pc[r] == len(progs[r]) for r in range(n)):
                return
            raise ProtocolFailure("deadlock")
        r = rng.choice(cands)
        kind, c, other = progs[r][pc[r]]
        e = c + 1
        if kind == "write":
            stage[other][par(e)][r] = c
            flag[other][r] = e
        else:
            got = stage[r][par(e)][other]
            if got != c:
                raise ProtocolFailure(f"rank {r} call {c} read call {got}'s partial of "
                                      f"rank {other}")
        pc[r] += 1


@pytest.mark.parametrize("n", [2, 4, 8])
def test_per_tile_flag_protocol_is_race_free(n):
    for seed in range(300):
        simulate(n, calls=4, seed=seed)


def test_single_staging_buffer_races():
    with pytest.raises(ProtocolFailure, match="read call"):
        for seed in range(300):
            simulate(2, calls=4, seed=seed, double_buffer=False)


def test_own_rows_first_deadlocks():
    with pytest.raises(ProtocolFailure, match="deadlock"):
        simulate(2, calls=1, seed=0, own_rows_last=False)
