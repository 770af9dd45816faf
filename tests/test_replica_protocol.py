"""Model check of the fused data-parallel step's signalling (pure Python, CPU).

The fused replica path (``data_parallel/replica_comm.py``, ``csrc/dp_comm.cu``) runs, on
every replica rank r and every step k, in stream order:

1. forward: reads every shard of r's own bf16 parameter buffer;
2. backward: writes every shard of r's own fp32 gradient buffer;
3. signal(GRAD): flag_grad[dst][r] = k + 1 for every dst;
4. replica_reduce: for every src != r, wait flag_grad[r][src] >= k + 1, then read src's
   gradient at r's shard (the reads of one kernel happen in any order); then write the
   sum into r's own gradient shard;
5. replica_adamw_gather: write r's updated parameter shard into every replica's
   parameter buffer (peer stores, any order);
6. signal(PARAM), then replica_wait: wait flag_param[r][src] >= k + 1 for every src.

A random scheduler interleaves the ranks' events, honouring stream order and the waits.
Invariants: a forward of step k reads only parameters of version k - 1 (no shard stale,
none from the future); a reduce of step k reads the peer's step-k local gradient (not yet
overwritten by the peer's next backward, not a peer's reduced value); every run
completes. Variants without the final wait, or without the GRAD wait, must be caught,
which shows the checker finds the races the protocol prevents.
"""

from __future__ import annotations

import random

import pytest


class ProtocolRace(AssertionError):
    pass


def _program(r: int, n: int, steps: int, *, param_wait: bool, grad_wait: bool) -> list:
    """Groups of events; the events of one group (one kernel) run in any order."""
    prog = []
    for k in range(steps):
        prog.append([("fwd_read", k, s) for s in range(n)])
        prog.append([("bwd_write", k, s) for s in range(n)])
        prog.append([("sig_grad", k)])
        prog.append([("reduce_read", k, src, grad_wait) for src in range(n) if src != r])
        prog.append([("reduce_write", k)])
        prog.append([("adam_write", k, dst) for dst in range(n)])
        prog.append([("sig_param", k)])
        if param_wait:
            prog.append([("wait_param", k)])
    return prog


def simulate(n: int, steps: int, seed: int, *, param_wait: bool = True,
             grad_wait: bool = True) -> None:
    rng = random.Random(seed)
    progs = [_program(r, n, steps, param_wait=param_wait, grad_wait=grad_wait)
             for r in range(n)]
    group = [0] * n                      # current group per rank
    done = [set() for _ in range(n)]     # indices of the current group already executed
    flag_grad = [[0] * n for _ in range(n)]     # [reader][writer]
    flag_param = [[0] * n for _ in range(n)]
    grad = [[("init", -1)] * n for _ in range(n)]   # [rank][shard] -> (kind, step)
    param = [[-1] * n for _ in range(n)]            # [rank][shard] -> version

    def ready(r, ev) -> bool:
        if ev[0] == "reduce_read":
            _, k, src, waits = ev
            return (not waits) or flag_grad[r][src] >= k + 1
        if ev[0] == "wait_param":
            return all(flag_param[r][src] >= ev[1] + 1 for src in range(n))
        return True

    def run(r, ev) -> None:
        kind = ev[0]
        if kind == "fwd_read":
            _, k, s = ev
            if param[r][s] != k - 1:
                raise ProtocolRace(f"rank {r} forward of step {k} read shard {s} at version "
                                   f"{param[r][s]}")
        elif kind == "bwd_write":
            _, k, s = ev
            grad[r][s] = ("local", k)
        elif kind == "sig_grad":
            for dst in range(n):
                flag_grad[dst][r] = ev[1] + 1
        elif kind == "reduce_read":
            _, k, src, _w = ev
            if grad[src][r] != ("local", k):
                raise ProtocolRace(f"rank {r} reduce of step {k} read {grad[src][r]} from "
                                   f"rank {src}")
        elif kind == "reduce_write":
            grad[r][r] = ("reduced", ev[1])
        elif kind == "adam_write":
            _, k, dst = ev
            param[dst][r] = k
        elif kind == "sig_param":
            for dst in range(n):
                flag_param[dst][r] = ev[1] + 1

    while True:
        cands = []
        for r in range(n):
            if group[r] >= len(progs[r]):
                continue
            for i, ev in enumerate(progs[r][group[r]]):
                if i not in done[r] and ready(r, ev):
                    cands.append((r, i, ev))
        if not cands:
            if all(group[r] >= len(progs[r]) for r in range(n)):
                return
            raise ProtocolRace("deadlock: no rank can make progress")
        r, i, ev = rng.choice(cands)
        run(r, ev)
        done[r].add(i)
        if len(done[r]) == len(progs[r][group[r]]):
            group[r] += 1
            done[r] = set()


@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_fused_replica_step_protocol_is_race_free(n):
    for seed in range(300):
        simulate(n, steps=3, seed=seed)


def test_dropping_the_parameter_wait_is_caught():
    with pytest.raises(ProtocolRace):
        for seed in range(300):
            simulate(2, steps=3, seed=seed, param_wait=False)


def test_dropping_the_gradient_wait_is_caught():
    with pytest.raises(ProtocolRace):
        for seed in range(300):
            simulate(2, steps=2, seed=seed, grad_wait=False)
