"""Fused AG->GEMM and GEMM->RS across real GPUs (IPC-mapped symmetric buffers, NCCL oracle).

Runs as child processes, one per GPU, over 2 GPUs when the box has them (skipped
otherwise). Every wait in the kernels is bounded; the process group has a short
timeout and the parent joins with a deadline.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _worker(rank, world, port, errq, rs_in_kernel=False):
    import traceback
    from datetime import timedelta

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        from types import SimpleNamespace

        from nano_megatron_b200.distributed.symmetric import SymmetricWorkspace
        from nano_megatron_b200.ops import comm_gemm as CG
        from nano_megatron_b200.ops._ext import status_word

        CG.RS_IN_KERNEL = rs_in_kernel    # reduce-scatter reduced in the GEMM epilogue
        grp = SimpleNamespace(rank=rank, size=world, process_group=dist.group.WORLD)
        ws = SymmetricWorkspace.create(grp, rs_bytes=32 << 20, ag_bytes=16 << 20, device=dev)
        R, K, N = 1024, 1024, 1024
        for it in range(4):
            g = torch.Generator(device=dev).manual_seed(100 * it + rank)
            a = torch.randn(R * world, K, device=dev, generator=g).bfloat16()
            w = torch.randn(N, K, device=dev, generator=g).bfloat16() * 0.05
            res = torch.randn(R, N, device=dev, generator=g).bfloat16()
            out = CG.gemm_reduce_scatter(ws, a, w, residual=res)
            part = (a.float() @ w.float().t())
            ref = torch.empty(R, N, device=dev)
            dist.reduce_scatter_tensor(ref, part)
            ref += res.float()
            err = ((out.float() - ref).norm() / ref.norm()).item()
            assert err < 1e-2, f"rs rank {rank} it {it}: {err}"
            x = torch.randn(R, K, device=dev, generator=g).bfloat16()
            wc = torch.randn(N, K, device=dev, generator=g).bfloat16() * 0.05
            y, xf = CG.allgather_gemm(ws, x, wc)
            xg = torch.empty(R * world, K, device=dev, dtype=torch.bfloat16)
            dist.all_gather_into_tensor(xg, x)
            assert torch.equal(xf, xg), f"gathered copy differs on rank {rank}"
            ref2 = xg.float() @ wc.float().t()
            err2 = ((y.float() - ref2).norm() / ref2.norm()).item()
            assert err2 < 1e-2, f"ag rank {rank} it {it}: {err2}"
        torch.cuda.synchronize()
        assert int(status_word(dev).item()) == 0
        dist.barrier(device_ids=[rank])
        ws.close()                        # unmap peers once nobody stores into them
        dist.barrier(device_ids=[rank])
        ws.release()                      # free the own buffer once no peer maps it
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise


@pytest.mark.parametrize("rs_in_kernel", [False, True], ids=["rs_two_pass", "rs_in_kernel"])
def test_fused_tp_collectives_two_gpus(rs_in_kernel):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    from dist_utils import free_port

    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, errq, rs_in_kernel))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    if not errq.empty():
        r, tb = errq.get()
        raise AssertionError(f"rank {r} failed:\n{tb}")
    assert not alive, "ranks timed out"
    assert all(p.exitcode == 0 for p in procs)
