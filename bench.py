"""Headline benchmark: device-timed training tokens/s of the 311M GPT.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Config (the reference's headline 311M config): 24 layers, hidden 1024, 16 MHA
heads of 64, SwiGLU 2736, vocab 8192 (310,821,888 parameters), seq 512, global
batch 256, micro-batch 8, bf16, AdamW lr 3e-4 cosine, clip 1.0, DDP bucketed
all-reduce. Layout by GPU count: 1 -> TP1, 2 -> TP2+SP, 4 -> TP2xPP2+SP (1F1B,
P2P overlap), 8 -> TP2xPP2xDP2+SP. Data: synthetic uniform-random token ids;
random-init weights.

``value`` is whole-job tokens/s from CUDA events around exactly K train steps
(barrier + synchronize on both sides, max over ranks). ``e2e`` repeats the K
steps through the public ``Trainer.train_step`` API with, every step, a
host->device copy of that step's token batch from pinned memory and a
device->host read of the step's loss. Activations and weights far exceed the
126 MB L2, so no explicit flush is done between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
MODEL = {"layers": 24, "hidden_size": 1024, "ffn_hidden_size": 2736, "heads": 16,
         "kv_heads": 16, "seq_length": 512, "vocab_size": 8192, "dropout": 0.0,
         "tie_embeddings": True}
GLOBAL_BATCH = 256
MICRO_BATCH = 8
LAYOUTS = {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 2, 2)}  # (tp, pp, dp)
BASELINE_PUBLISHED = None  # the reference publishes no throughput number


def make_config_dict(n_gpus: int, steps: int) -> dict:
    tp, pp, dp = LAYOUTS[n_gpus]
    gas = GLOBAL_BATCH // (MICRO_BATCH * dp)
    return {
        "distributed": {"backend": "nccl", "device": "cuda", "timeout_minutes": 10},
        "parallel": {"tensor": tp, "pipeline": pp, "context": 1, "expert": 1, "data": dp,
                     "order": ["tp", "cp", "ep", "dp", "pp"], "sequence_parallel": tp > 1},
        "model": dict(MODEL),
        "precision": {"params": "bfloat16", "compute": "bfloat16", "grad_reduce": "float32"},
        "data_parallel": {"mode": "ddp", "bucket_bytes": 268435456,
                          "overlap_grad_reduce": True},
        "pipeline": {"schedule": "1f1b", "overlap_p2p": True},
        "optimizer": {"lr": 3e-4, "betas": [0.9, 0.95], "eps": 1e-8, "weight_decay": 0.1,
                      "clip_grad_norm": 1.0},
        "lr_scheduler": {"schedule": "cosine", "warmup_steps": 0,
                         "decay_steps": max(10488, steps + 100), "min_lr": 3e-5},
        "training": {"micro_batch_size": MICRO_BATCH, "gradient_accumulation_steps": gas,
                     "max_steps": max(10488, steps + 100), "seed": 1234, "log_interval": 10},
    }


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu),
                                      f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        sm = sorted(float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit())
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) > 8:
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


# ---------------------------------------------------------------------- common
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def synthetic_batches(n: int, rows: int, seq: int, vocab: int, seed: int):
    import torch

    gen = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, vocab, (rows, seq + 1), generator=gen)
        out.append({"input_ids": ids[:, :-1].contiguous().pin_memory(),
                    "labels": ids[:, 1:].contiguous().pin_memory()})
    return out


def barrier_sync(device):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize(device)
    if dist.is_available() and dist.is_initialized():
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


def max_over_ranks(x: float, device) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_timed(trainer, batches, steps: int, warmup: int, device, is_source: bool, *,
              e2e: bool, lib=None):
    """Warm up, then time exactly ``steps`` train steps with CUDA events."""
    import torch

    def step(i):
        b = batches[i % len(batches)] if is_source else None
        if not e2e and is_source:
            b = staged[i % len(staged)]
        out = trainer.train_step(b)
        if e2e:
            loss = out["loss_sum"] if isinstance(out, dict) else out.metrics.get("loss")
            if isinstance(loss, torch.Tensor):
                _ = float(loss.detach().to("cpu"))
        return out

    staged = [{k: v.to(device, non_blocking=True) for k, v in b.items()} for b in batches] \
        if (is_source and not e2e) else []
    for i in range(warmup):
        step(i)
    barrier_sync(device)
    launches0 = lib.launch_count() if lib is not None else 0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    t0 = time.perf_counter()
    for i in range(steps):
        step(warmup + i)
    end.record()
    barrier_sync(device)
    wall = time.perf_counter() - t0
    ms = start.elapsed_time(end)
    launches = (lib.launch_count() - launches0) if lib is not None else None
    return max_over_ranks(ms, device), max_over_ranks(wall * 1000.0, device), launches


# ---------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local):
    sys.path.insert(0, ROOT)
    import torch

    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.ops import _ext
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    d = make_config_dict(args.gpus, args.steps + args.warmup)
    d["kernels"] = {"backend": "b200", "fused_tp_comm": not args.no_fused_tp,
                    "cuda_graphs": not args.no_cuda_graphs}
    cfg = config_from_dict(d)
    runtime = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, runtime)
    device = runtime.device
    trainer = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                      data_parallel=comps.data_parallel, rng=comps.rng, device=device)
    dp = comps.parallel.dp.size
    rows = GLOBAL_BATCH // dp
    batches = synthetic_batches(4, rows, MODEL["seq_length"], MODEL["vocab_size"],
                                seed=1234 + comps.parallel.coordinate.dp)
    src = trainer.batch_router.is_source
    lib = _ext.lib()
    with ClockSampler(local) as clocks:
        dev_ms, _, launches = run_timed(trainer, batches, args.steps, args.warmup, device, src,
                                        e2e=False, lib=lib)
    e2e_ms, e2e_wall, _ = run_timed(trainer, batches, args.steps, 0, device, src, e2e=True)
    _ext.check_status(device)
    return finish(args, rank, world, dev_ms, e2e_ms, e2e_wall, clocks.summary(), launches,
                  impl="ours", runtime=runtime)


# ---------------------------------------------------------------------- reference arm
def run_reference(args, rank, world, local):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nano_megatron")):
        return unavailable("reference not installed in baseline/_ref")
    sys.path.insert(0, ref)
    import torch

    from nano_megatron.config import config_from_dict
    from nano_megatron.data_parallel import build_data_parallel_strategy
    from nano_megatron.distributed import DistributedRuntime
    from nano_megatron.models.gpt import DenseGPTComponents, GPTModelBuilder
    from nano_megatron.nn.kernels import build_kernel_backend
    from nano_megatron.context_parallel import build_context_parallel_attention
    from nano_megatron.parallel import ParallelContext, ParallelRNG, ParameterDomainRegistry, RNGStream
    from nano_megatron.training import Trainer

    d = make_config_dict(args.gpus, args.steps + args.warmup)
    d["wandb"] = {"enabled": False}
    cfg = config_from_dict(d)
    runtime = DistributedRuntime(cfg.distributed).initialize()
    parallel = ParallelContext.create(runtime, cfg.parallel)
    rng = ParallelRNG.from_context(cfg.training.seed, parallel)
    torch.manual_seed(rng.seed(RNGStream.DENSE_INIT))
    kernels = build_kernel_backend(cfg.kernels, parallel)
    cp_attention = build_context_parallel_attention(cfg.context_parallel, parallel)
    builder = GPTModelBuilder(DenseGPTComponents(cp_attention=cp_attention),
                              parameter_domains=ParameterDomainRegistry(),
                              activation_checkpoint_config=cfg.activation_checkpoint)
    built = builder.build_stage(cfg.model, parallel, kernels, rng=rng)
    dtype = {"bfloat16": torch.bfloat16, "float32": torch.float32}[cfg.precision.params.value]
    model = built.model.to(device=runtime.device, dtype=dtype)
    strategy = build_data_parallel_strategy(cfg.data_parallel, cfg.offload, parallel,
                                            built.parameter_domains)
    trainer = Trainer(config=cfg, model=model, parallel=parallel, data_parallel=strategy,
                      rng=rng)
    device = runtime.device
    rows = GLOBAL_BATCH // parallel.dp.size
    batches = synthetic_batches(4, rows, MODEL["seq_length"], MODEL["vocab_size"],
                                seed=1234 + parallel.coordinate.dp)
    src = trainer.batch_router.is_source
    with ClockSampler(local) as clocks:
        dev_ms, _, _ = run_timed(trainer, batches, args.steps, args.warmup, device, src, e2e=False)
    e2e_ms, e2e_wall, _ = run_timed(trainer, batches, args.steps, 0, device, src, e2e=True)
    return finish(args, rank, world, dev_ms, e2e_ms, e2e_wall, clocks.summary(), None,
                  impl="reference", runtime=runtime)


def unavailable(why: str) -> int:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
    return 0


def finish(args, rank, world, dev_ms, e2e_ms, e2e_wall_ms, clocks, launches, *, impl, runtime):
    tokens_per_step = GLOBAL_BATCH * MODEL["seq_length"]
    value = tokens_per_step * args.steps / (dev_ms / 1000.0)
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)
    tp, pp, dp = LAYOUTS[args.gpus]
    layout = "".join(f"{n}{s}" for n, s in (("tp", tp), ("pp", pp), ("dp", dp)) if s > 1) or "tp1"
    line = {
        "metric": "tokens/sec (device-timed, max over ranks) for 311M TP2xPP2xDP2 at 1/2/4/8 B200",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None if BASELINE_PUBLISHED is None else value / BASELINE_PUBLISHED,
        "dtype": "bf16", "data": "synthetic uniform-random token ids, random-init weights",
        "config": {"model": "GPT-311M (24L, H1024, 16 heads, F2736, V8192, tied)",
                   "global_batch": GLOBAL_BATCH, "seq_len": MODEL["seq_length"],
                   "micro_batch": MICRO_BATCH, "parallelism": layout,
                   "l2": "no flush: weights (622 MB) and activations exceed the 126 MB L2"},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "wall_ms_per_step": e2e_wall_ms / args.steps,
                "h2d_bytes_per_step": 2 * (GLOBAL_BATCH // dp) * MODEL["seq_length"] * 8,
                "d2h_bytes_per_step": 8},
        "impl": impl,
    }
    if launches is not None:
        line["gpu_launches"] = launches
    if rank == 0:
        print(json.dumps(line), flush=True)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    runtime.close()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1, choices=sorted(LAYOUTS))
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-fused-tp", action="store_true",
                    help="diagnostic: NCCL all-gather/reduce-scatter instead of the fused "
                         "NVLink AG->GEMM / GEMM->RS kernels")
    ap.add_argument("--no-cuda-graphs", action="store_true",
                    help="diagnostic: launch every kernel from Python instead of replaying one "
                         "CUDA graph per microbatch")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    if args.impl == "reference":
        return run_reference(args, rank, world, local)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
