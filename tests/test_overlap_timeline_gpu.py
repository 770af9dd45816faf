"""Timeline check on two GPUs: the DDP bucket all-reduce overlaps backward compute.

Like the reference's profiler timeline tests (tests/distributed_gpu/test_pipeline_overlap_nccl.py:
730-824), this one is opt-in (``NMB_RUN_TIMELINE_TESTS=1``): it records one training step
of a DP2 run with ``torch.profiler``, and requires an NCCL kernel to run concurrently with
this framework's GEMM kernels for at least 100 us in total. Child processes, one per GPU,
bounded by timeouts, NVLS off.
"""

import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _cfg():
    from nano_megatron_b200.config import config_from_dict

    return config_from_dict({
        "distributed": {"backend": "nccl", "device": "cuda", "timeout_minutes": 2},
        "parallel": {"tensor": 1, "pipeline": 1, "context": 1, "expert": 1, "data": WORLD},
        "model": {"layers": 8, "hidden_size": 1024, "ffn_hidden_size": 2736, "heads": 16,
                  "kv_heads": 16, "seq_length": 512, "vocab_size": 8192},
        "precision": {"params": "bfloat16", "compute": "bfloat16", "grad_reduce": "float32"},
        "kernels": {"backend": "b200"},
        "data_parallel": {"mode": "ddp", "overlap_grad_reduce": True,
                          "bucket_bytes": 16 * 1024 * 1024},
        "training": {"micro_batch_size": 8, "gradient_accumulation_steps": 2, "seed": 3},
        "optimizer": {"lr": 1e-4}})


def _intervals(trace: dict, pred) -> list:
    out = []
    for ev in trace.get("traceEvents", []):
        if ev.get("ph") == "X" and ev.get("cat") == "kernel" and pred(ev.get("name", "")):
            out.append((float(ev["ts"]), float(ev["ts"]) + float(ev.get("dur", 0.0))))
    return sorted(out)


def _overlap_us(a: list, b: list) -> float:
    total = 0.0
    for s0, e0 in a:
        for s1, e1 in b:
            total += max(0.0, min(e0, e1) - max(s0, s1))
    return total


def _worker(rank, world, port, out_dir, errq):
    import traceback

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        from nano_megatron_b200.distributed import DistributedRuntime
        from nano_megatron_b200.training import Trainer
        from nano_megatron_b200.training.engine import build_training_components

        cfg = _cfg()
        runtime = DistributedRuntime(cfg.distributed).initialize()
        comps = build_training_components(cfg, runtime)
        tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                     data_parallel=comps.data_parallel, rng=comps.rng)
        g = torch.Generator().manual_seed(rank)
        ids = torch.randint(0, 8192, (16, 513), generator=g)
        batch = {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous()}
        for _ in range(3):
            tr.train_step(batch)
        torch.cuda.synchronize()
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU,
                                                torch.profiler.ProfilerActivity.CUDA]) as prof:
            tr.train_step(batch)
            torch.cuda.synchronize()
        path = os.path.join(out_dir, f"trace{rank}.json")
        prof.export_chrome_trace(path)
        comps.close(tr)
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise


@pytest.mark.skipif(os.environ.get("NMB_RUN_TIMELINE_TESTS") != "1",
                    reason="timeline test is opt-in: NMB_RUN_TIMELINE_TESTS=1")
def test_ddp_all_reduce_overlaps_backward_gemms(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    from dist_utils import free_port

    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, str(tmp_path), errq))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    if not errq.empty():
        r, tb = errq.get()
        raise AssertionError(f"rank {r} failed:\n{tb}")
    assert not alive and all(p.exitcode == 0 for p in procs)
    trace = json.loads((tmp_path / "trace0.json").read_text())
    nccl = _intervals(trace, lambda n: "nccl" in n.lower())
    gemm = _intervals(trace, lambda n: "gemm_tcgen05" in n)
    assert nccl and gemm, (len(nccl), len(gemm))
    assert _overlap_us(nccl, gemm) >= 100.0, _overlap_us(nccl, gemm)
