"""Validate and time NCCL collectives and ring P2P under ``torchrun`` (``nano-megatron-validate-nccl``).

Checks correctness (all-reduce of rank ids, all-gather of rank ids, ring
payloads), then times all-reduce, all-gather, reduce-scatter and a
send/receive ring with CUDA events on the issuing stream after warm-up, taking
the maximum over ranks; prints one JSON report with algorithm and bus
bandwidths (bus factor 2(n-1)/n for all-reduce, (n-1)/n for the gather and
scatter). Counterpart of the reference's scripts/validate_nccl.py, which times
with host clocks.
"""

from __future__ import annotations

import argparse
import json
import os
from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--collective-mib", type=int, default=256)
    p.add_argument("--all-gather-mib", type=int, default=32, help="per-rank shard size")
    p.add_argument("--p2p-mib", type=int, default=256)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iterations", type=int, default=20)
    p.add_argument("--barrier-iterations", type=int, default=200)
    p.add_argument("--timeout-s", type=float, default=120.0)
    return p


def _pos(name: str, v: int) -> int:
    if isinstance(v, bool) or not isinstance(v, int) or v < 1:
        raise ValueError(f"{name} must be a positive integer")
    return v


def device_time_ms(op: Callable[[], None], *, warmup: int, iters: int,
                   device: torch.device) -> float:
    """Mean device milliseconds per call, max over ranks."""
    for _ in range(warmup):
        op()
    torch.cuda.synchronize(device)
    dist.barrier(device_ids=[device.index])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        op()
    b.record()
    torch.cuda.synchronize(device)
    t = torch.tensor(a.elapsed_time(b) / iters, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _gbs(nbytes: int, ms: float, factor: float = 1.0) -> float:
    return nbytes * factor / (ms * 1e-3) / 1e9


def main(argv: Sequence[str] | None = None) -> None:
    from datetime import timedelta

    a = parser().parse_args(argv)
    warm, iters = _pos("warmup", a.warmup), _pos("iterations", a.iterations)
    bar_iters = _pos("barrier_iterations", a.barrier_iterations)
    rank, local, world = (int(os.environ[k]) for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE"))
    if not torch.cuda.is_available() or not dist.is_nccl_available():
        raise RuntimeError("validate_nccl requires CUDA and NCCL")
    if world < 2:
        raise ValueError("validate_nccl requires at least two ranks")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=a.timeout_s))
    try:
        x = torch.tensor(float(rank + 1), device=dev)
        dist.all_reduce(x)
        if float(x) != world * (world + 1) / 2:
            raise RuntimeError(f"all-reduce correctness failed on rank {rank}: {float(x)}")
        ids = torch.empty(world, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(ids, torch.tensor([rank], dtype=torch.int64, device=dev))
        if ids.tolist() != list(range(world)):
            raise RuntimeError(f"all-gather correctness failed on rank {rank}: {ids.tolist()}")
        mib = 1 << 20
        ar = torch.zeros(a.collective_mib * mib // 2, dtype=torch.bfloat16, device=dev)
        ar_ms = device_time_ms(lambda: dist.all_reduce(ar), warmup=warm, iters=iters, device=dev)
        shard = torch.full((a.all_gather_mib * mib // 2,), float(rank), dtype=torch.bfloat16,
                           device=dev)
        full = torch.empty(world * shard.numel(), dtype=shard.dtype, device=dev)
        ag_ms = device_time_ms(lambda: dist.all_gather_into_tensor(full, shard), warmup=warm,
                               iters=iters, device=dev)
        for r, part in enumerate(full.view(world, -1)):
            if not bool((part == float(r)).all()):
                raise RuntimeError(f"timed all-gather payload failed on rank {rank} from {r}")
        rs_out = torch.empty_like(shard)
        rs_ms = device_time_ms(lambda: dist.reduce_scatter_tensor(rs_out, full), warmup=warm,
                               iters=iters, device=dev)
        send = torch.full((a.p2p_mib * mib // 2,), float(rank), dtype=torch.bfloat16, device=dev)
        recv = torch.empty_like(send)
        prev, nxt = (rank - 1) % world, (rank + 1) % world

        def ring() -> None:
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, send, nxt),
                                             dist.P2POp(dist.irecv, recv, prev)]):
                w.wait()

        p2p_ms = device_time_ms(ring, warmup=warm, iters=iters, device=dev)
        if not bool((recv == float(prev)).all()):
            raise RuntimeError(f"ring P2P payload failed on rank {rank}: expected {prev}")
        bar_ms = device_time_ms(lambda: dist.barrier(device_ids=[local]), warmup=warm,
                                iters=bar_iters, device=dev)
        if rank == 0:
            n = world
            out = {"world_size": n, "device": torch.cuda.get_device_name(dev),
                   "torch": torch.__version__, "cuda": torch.version.cuda,
                   "nccl": list(torch.cuda.nccl.version()), "iterations": iters,
                   "timing": "cuda events on the issuing stream, mean per call, max over ranks",
                   "all_reduce": {"payload_mib": a.collective_mib, "ms": ar_ms,
                                  "algo_gbs": _gbs(ar.numel() * 2, ar_ms),
                                  "bus_gbs": _gbs(ar.numel() * 2, ar_ms, 2 * (n - 1) / n)},
                   "all_gather": {"shard_mib": a.all_gather_mib, "ms": ag_ms,
                                  "bus_gbs": _gbs(full.numel() * 2, ag_ms, (n - 1) / n)},
                   "reduce_scatter": {"shard_mib": a.all_gather_mib, "ms": rs_ms,
                                      "bus_gbs": _gbs(full.numel() * 2, rs_ms, (n - 1) / n)},
                   "p2p_ring": {"payload_mib": a.p2p_mib, "ms": p2p_ms,
                                "gbs_per_direction": _gbs(send.numel() * 2, p2p_ms)},
                   "barrier": {"iterations": bar_iters, "us": bar_ms * 1e3}}
            print(json.dumps(out, sort_keys=True))
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
