"""Fused compute + collective paths over NVLink peer memory, timed against NCCL.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m nano_megatron_b200.ops.bench_comm [--case all|tp|replica] [--iters K]

Every rank runs the same sequence; each case is timed with CUDA events on the launching
stream after warm-up, bracketed by a barrier and a synchronize, and the reported time is
the maximum over ranks. For each fused path the line gives its FLOPs, the bytes it must
move over NVLink per rank (one direction), the roofline time -- the slower of FLOPs at
the measured bf16 GEMM peak and those bytes at the measured 770 GB/s peer-copy bandwidth
(an HBM term is added where the path is memory-bound: bytes at the measured copy
bandwidth) -- and achieved = roofline / measured. The NCCL equivalent (library
collective + the same local kernels) is timed beside it.

Cases (shapes of the 311M model under TP2 with a 64-sequence micro-batch, and of its
8-GPU data-parallel replica group):
* ``tp_rs``  GEMM -> reduce-scatter (out_proj forward, sequence parallel): peer-store
  epilogue + flag-gated reduce kernel on the owner (``ops.comm_gemm.gemm_reduce_scatter``),
  and the opt-in variant that reduces this rank's rows in the GEMM's own epilogue, vs
  GEMM + ``reduce_scatter_tensor``.
* ``tp_ag``  all-gather -> GEMM (QKV forward): gathered-A GEMM reading peer shards
  (``ops.comm_gemm.allgather_gemm``) vs ``all_gather_into_tensor`` + GEMM.
* ``replica`` DDP / ZeRO-1/2 step: replica reduce of this rank's fp32 gradient shard
  from every peer + sharded AdamW + bf16 parameter stores into every replica
  (``data_parallel.replica_comm``) vs ``all_reduce`` + AdamW over the whole buffer.

Reference behaviour these paths replace: src/nano_megatron/tensor_parallel/layers.py
(sequence-parallel all-gather / reduce-scatter around F.linear),
src/nano_megatron/data_parallel/buckets.py:210-303 (bucket all-reduce) and
src/nano_megatron/data_parallel/_zero.py:166-199 (reduce-scatter, AdamW, all-gather).
"""

from __future__ import annotations

import argparse
import json
import math
import os
from datetime import timedelta
from types import SimpleNamespace

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0   # measured peer copy per direction on this pool's B200s


def _peaks() -> tuple[float, float]:
    """(bf16 TFLOP/s burst, HBM GB/s) from MEASURED_PEAKS.json at the repository root."""
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def _timed(fn, iters: int, dev) -> float:
    """Mean ms per call, max over ranks (CUDA events; barrier + synchronize around)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier(device_ids=[dev.index])
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([s.elapsed_time(e) / iters], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    dist.barrier(device_ids=[dev.index])
    return float(ms.item())


def _line(name, fused_ms, nccl_ms, flops, link_bytes, hbm_bytes=0.0, **extra) -> dict:
    tflops, hbm_gbs = _peaks()
    t_compute = flops / (tflops * 1e12) * 1e3
    t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
    t_hbm = hbm_bytes / (hbm_gbs * 1e9) * 1e3
    roof = max(t_compute, t_link, t_hbm)
    return {"case": name, "fused_ms": round(fused_ms, 4), "nccl_ms": round(nccl_ms, 4),
            "speedup_vs_nccl": round(nccl_ms / fused_ms, 3), "gflop": round(flops / 1e9, 2),
            "nvlink_mb_per_rank": round(link_bytes / 1e6, 2),
            "hbm_mb": round(hbm_bytes / 1e6, 2), "roofline_ms": round(roof, 4),
            "bound": max((t_compute, "compute"), (t_link, "nvlink"), (t_hbm, "hbm"))[1],
            "achieved_frac_of_roofline": round(roof / fused_ms, 3), **extra}


def case_tp(grp, dev, iters: int, rows_total: int = 32768, hidden: int = 1024) -> list[dict]:
    from nano_megatron_b200.distributed.symmetric import SymmetricWorkspace
    from nano_megatron_b200.ops import comm_gemm as CG
    from nano_megatron_b200.ops import gemm as G

    n, r = grp.size, grp.rank
    rows = rows_total // n
    k_out = hidden // n                   # out_proj input features per rank (local heads)
    n_qkv = 3 * hidden // n               # QKV output features per rank
    ws = SymmetricWorkspace.create(grp, rs_bytes=rows * hidden * 2 * n,
                                   ag_bytes=rows * hidden * 2, device=dev)
    g = torch.Generator(device=dev).manual_seed(1 + r)
    out = []
    try:
        # --- GEMM -> reduce-scatter (out_proj): a [rows_total, k_out] x w [hidden, k_out]
        a = torch.randn(rows_total, k_out, device=dev, generator=g).bfloat16()
        w = (torch.randn(hidden, k_out, device=dev, generator=g) * 0.05).bfloat16()
        res = torch.randn(rows, hidden, device=dev, generator=g).bfloat16()
        y = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16)
        full = torch.empty(rows_total, hidden, device=dev, dtype=torch.bfloat16)
        fused = _timed(lambda: CG.gemm_reduce_scatter(ws, a, w, residual=res, out=y), iters, dev)

        def nccl_rs():
            G.gemm(a, w, full)
            dist.reduce_scatter_tensor(y, full, group=grp.process_group)
            y.add_(res)
        base = _timed(nccl_rs, iters, dev)
        flops = 2.0 * rows_total * hidden * k_out
        link = (n - 1) / n * rows_total * hidden * 2.0
        out.append(_line("tp_rs_out_proj", fused, base, flops, link,
                         shape=f"{rows_total}x{hidden}x{k_out}", tp=n,
                         reduction="second kernel on the owner"))
        saved, CG.RS_IN_KERNEL = CG.RS_IN_KERNEL, True   # the opt-in variant
        try:
            t2 = _timed(lambda: CG.gemm_reduce_scatter(ws, a, w, residual=res, out=y), iters,
                        dev)
        finally:
            CG.RS_IN_KERNEL = saved
        out.append(_line("tp_rs_out_proj_in_kernel", t2, base, flops, link,
                         shape=f"{rows_total}x{hidden}x{k_out}", tp=n,
                         reduction="in the GEMM epilogue (NMB_RS_IN_KERNEL=1)"))
        # --- all-gather -> GEMM (QKV): x_local [rows, hidden] x w [n_qkv, hidden]
        x = torch.randn(rows, hidden, device=dev, generator=g).bfloat16()
        wq = (torch.randn(n_qkv, hidden, device=dev, generator=g) * 0.05).bfloat16()
        q = torch.empty(rows_total, n_qkv, device=dev, dtype=torch.bfloat16)
        xg = torch.empty(rows_total, hidden, device=dev, dtype=torch.bfloat16)
        fused = _timed(lambda: CG.allgather_gemm(ws, x, wq), iters, dev)

        def nccl_ag():
            dist.all_gather_into_tensor(xg, x, group=grp.process_group)
            G.gemm(xg, wq, q)
        base = _timed(nccl_ag, iters, dev)
        flops = 2.0 * rows_total * n_qkv * hidden
        link = (n - 1) / n * rows_total * hidden * 2.0
        out.append(_line("tp_ag_qkv", fused, base, flops, link,
                         shape=f"{rows_total}x{n_qkv}x{hidden}", tp=n))
        torch.cuda.synchronize(dev)
        from nano_megatron_b200.ops._ext import status_word

        assert int(status_word(dev).item()) == 0, "a bounded peer wait timed out"
    finally:
        dist.barrier(device_ids=[dev.index])
        ws.close()
        dist.barrier(device_ids=[dev.index])
        ws.release()
    return out


def case_replica(grp, dev, iters: int, numel: int = 78_000_000) -> list[dict]:
    from nano_megatron_b200.data_parallel.replica_comm import CH_GRAD, CH_PARAM, ReplicaComm
    from nano_megatron_b200.ops._ext import lib, status_word

    n, r = grp.size, grp.rank
    shard = math.ceil(numel / n)
    padded = shard * n
    rc = ReplicaComm.create(grp, padded, torch.bfloat16, torch.float32, dev)
    out = []
    try:
        params, grads = rc.flat_tensors(padded, torch.bfloat16, torch.float32)
        g = torch.Generator(device=dev).manual_seed(7 + r)
        grads.copy_(torch.randn(padded, device=dev, generator=g) * 1e-3)
        master = torch.randn(shard, device=dev, generator=g)
        m = torch.zeros(shard, device=dev)
        v = torch.zeros(shard, device=dev)
        bucket = SimpleNamespace(index=0, rank=r, shard_numel=shard,
                                 slices=[SimpleNamespace(start=0, end=padded)])
        rc.prepare(SimpleNamespace(device=dev, buckets=[bucket]), lambda s: True)
        off = lambda b: 0  # noqa: E731

        def fused():
            rc.signal(CH_GRAD)
            rc.reduce(bucket, off)
            rc.adamw_gather(bucket, off, master, m, v, lr=1e-4, betas=(0.9, 0.95), eps=1e-8,
                            wd=0.1, step=1, grad_scale=None, lr_t=None)
            rc.signal(CH_PARAM)
            rc.wait(CH_PARAM)
        t_fused = _timed(fused, iters, dev)
        # NCCL equivalent (DDP): all-reduce the fp32 gradients, AdamW over the whole buffer
        g2 = torch.randn(padded, device=dev, generator=g) * 1e-3
        master_f = torch.randn(padded, device=dev, generator=g)
        mf, vf = torch.zeros(padded, device=dev), torch.zeros(padded, device=dev)
        pf = torch.empty(padded, device=dev, dtype=torch.bfloat16)

        def nccl():
            dist.all_reduce(g2, group=grp.process_group)
            lib().adamw_step(master_f, g2, mf, vf, pf, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1, None, None)
        t_nccl = _timed(nccl, iters, dev)
        torch.cuda.synchronize(dev)
        assert int(status_word(dev).item()) == 0, "a bounded peer wait timed out"
        link = (n - 1) * shard * 4.0 + (n - 1) * shard * 2.0   # gradient loads + bf16 stores
        hbm = shard * (4.0 * n + 4 * 2 + 8 * 2 + 2.0 * n)      # grads, master, moments, params
        out.append(_line("replica_ddp_step", t_fused, t_nccl, 0.0, link, hbm,
                         numel=padded, replicas=n))
    finally:
        dist.barrier(device_ids=[dev.index])
        rc.close()
        dist.barrier(device_ids=[dev.index])
        rc.release()
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["all", "tp", "replica"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--numel", type=int, default=78_000_000)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    grp = SimpleNamespace(rank=rank, size=world, process_group=dist.group.WORLD)
    lines = []
    try:
        if a.case in ("all", "tp"):
            lines += case_tp(grp, dev, a.iters)
        if a.case in ("all", "replica"):
            lines += case_replica(grp, dev, a.iters, a.numel)
        if rank == 0:
            for ln in lines:
                print(json.dumps(ln), flush=True)
    finally:
        dist.barrier(device_ids=[dev.index])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
