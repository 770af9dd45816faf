"""Multi-process CPU (gloo) test harness: spawn ranks with a file rendezvous."""

from __future__ import annotations

import os
import tempfile
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _entry(rank, world, init_file, fn, args, errq):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "GLOO_SOCKET_IFNAME": "lo"})
    try:
        torch.set_num_threads(1)
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank,
                                world_size=world)
        fn(rank, world, *args)
        dist.barrier()
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(world: int, fn, *args, timeout: float = 300.0) -> None:
    """Run ``fn(rank, world, *args)`` on ``world`` gloo ranks; re-raise the first failure."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "rdzv")
        procs = [ctx.Process(target=_entry, args=(r, world, init_file, fn, args, errq))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        errors = []
        while not errq.empty():
            errors.append(errq.get())
        if errors:
            raise AssertionError("rank %d failed:\n%s" % errors[0])
        if alive:
            raise AssertionError(f"{len(alive)} rank(s) timed out")
        bad = [p.exitcode for p in procs if p.exitcode != 0]
        if bad:
            raise AssertionError(f"rank exit codes {bad}")


def _gpu_entry(rank, world, port, fn, args, errq):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "NCCL_NVLS_ENABLE": "0"})
    try:
        fn(rank, world, *args)
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def free_port() -> int:
    """A TCP port on 127.0.0.1 that nothing listens on right now, chosen by the OS (a
    fixed random range collides when several tests or workers start rendezvous at once)."""
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_gpu_ranks(world: int, fn, *args, timeout: float = 300.0) -> None:
    """Run ``fn(rank, world, *args)`` as one process per GPU (rank r on cuda:r) with the
    torchrun environment set (NCCL rendezvous on 127.0.0.1, NVLS off); ``fn`` initialises
    its own process group. Re-raises the first failure; kills ranks that outlive
    ``timeout``."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_gpu_entry, args=(r, world, port, fn, args, errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    if not errq.empty():
        raise AssertionError("rank %d failed:\n%s" % errq.get())
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) timed out")
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"rank exit codes {bad}")
