"""Headline benchmark: device-timed training tokens/s of the 311M GPT.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 311m|1p3b-cp|1p3b-zero1|1p3b-zero2|1p3b-zero3|8b]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Default config (the reference's headline 311M config): 24 layers, hidden 1024, 16
MHA heads of 64, SwiGLU 2736, vocab 8192 (310,821,888 parameters), seq 512, global
batch 256, micro-batch 8, bf16, AdamW lr 3e-4 cosine, clip 1.0, DDP bucketed
all-reduce. Layout by GPU count: 1 -> TP1, 2 -> TP2+SP, 4 -> TP2xPP2+SP (1F1B,
P2P overlap), 8 -> TP2xPP2xDP2+SP. Data: synthetic uniform-random token ids;
random-init weights. ``--config`` selects the other benchmark configs of the
project (1.3B ring-CP at 32k tokens, 1.3B ZeRO-1/2/3, the 8B shape under
TP4xPP2 interleaved 1F1B with full activation checkpointing); ``WORKLOADS``
lists their layouts per GPU count. All use a fixed global batch (strong scaling).

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
METRIC = "tokens/sec (device-timed, max over ranks) for {} at 1/2/4/8 B200"
_L1P3B = {"layers": 24, "hidden_size": 2048, "ffn_hidden_size": 5504, "heads": 16,
          "kv_heads": 4, "vocab_size": 8192, "dropout": 0.0, "tie_embeddings": True}


def _zero(mode: str) -> dict:
    return {
        "title": "1.3B DP8 " + mode.upper(),
        "describe": f"GPT-1.3B (24L, H2048, 16 q / 4 kv heads of 128, F5504, V8192), {mode}",
        "model": dict(_L1P3B, seq_length=2048), "global_batch": 128, "micro_batch": 4,
        "layouts": {n: {"data": n} for n in (1, 2, 4, 8)},
        "sections": {"data_parallel": {"mode": mode, "overlap_grad_reduce": True}},
        # the reference keeps fp32 masters under FSDP2 only with fp32 parameters
        "reference_sections": {"precision": {"params": "float32", "compute": "bfloat16"}}
        if mode == "zero3" else {},
    }


# The benchmark configs. ``layouts`` maps GPU count -> parallel sizes; the global batch is
# fixed across GPU counts (strong scaling), so gradient accumulation = global / (mb * dp).
WORKLOADS = {
    "311m": {
        "title": "311M TP2\u00d7PP2\u00d7DP2",   # the headline metric's name, verbatim
        "describe": "GPT-311M (24L, H1024, 16 heads, F2736, V8192, tied)",
        "model": {"layers": 24, "hidden_size": 1024, "ffn_hidden_size": 2736, "heads": 16,
                  "kv_heads": 16, "seq_length": 512, "vocab_size": 8192, "dropout": 0.0,
                  "tie_embeddings": True},
        # micro-batch per GPU count (both arms): the largest that measured fastest at that
        # layout on B200 (fewer, larger GEMMs; PP keeps >= 16 microbatches in flight)
        "global_batch": 256, "micro_batch": {1: 32, 2: 64, 4: 32, 8: 32},
        "layouts": {1: {}, 2: {"tensor": 2}, 4: {"tensor": 2, "pipeline": 2},
                    8: {"tensor": 2, "pipeline": 2, "data": 2}},
        "sections": {"pipeline": {"schedule": "1f1b", "overlap_p2p": True},
                     "data_parallel": {"mode": "ddp", "overlap_grad_reduce": True}},
    },
    "1p3b-cp": {
        "title": "1.3B TP2xCP4 seq 32768",
        "describe": "GPT-1.3B (24L, H2048, 16 q / 4 kv heads of 128, F5504, V8192), "
                    "ring CP with load-balanced chunks",
        "model": dict(_L1P3B, seq_length=32768), "global_batch": 8, "micro_batch": 1,
        "layouts": {1: {}, 2: {"context": 2}, 4: {"tensor": 2, "context": 2},
                    8: {"tensor": 2, "context": 4}},
        "sections": {"context_parallel": {"backend": "ring", "load_balance": True},
                     "data_parallel": {"mode": "ddp", "overlap_grad_reduce": True}},
        # the reference has no load-balanced chunking (contiguous CP shards)
        "reference_sections": {"context_parallel": {"backend": "ring"}},
    },
    "1p3b-zero1": _zero("zero1"),
    "1p3b-zero2": _zero("zero2"),
    "1p3b-zero3": _zero("zero3"),
    "8b": {
        "title": "8B-shape TP4xPP2 interleaved",
        "describe": "Llama-style 8B shape (32L, H4096, 32 q / 8 kv heads of 128, F14336, "
                    "V32768, untied, rope 5e5), full activation checkpointing",
        "model": {"layers": 32, "hidden_size": 4096, "ffn_hidden_size": 14336, "heads": 32,
                  "kv_heads": 8, "seq_length": 4096, "vocab_size": 32768, "dropout": 0.0,
                  "rope_theta": 500000.0, "tie_embeddings": False},
        "global_batch": 64, "micro_batch": 1,
        # 8B with fp32 masters and Adam moments does not fit one 180 GB GPU
        "layouts": {2: {"tensor": 2}, 4: {"tensor": 4},
                    8: {"tensor": 4, "pipeline": 2, "virtual": 2}},
        "sections": {"activation_checkpoint": {"mode": "full"},
                     "data_parallel": {"mode": "ddp", "overlap_grad_reduce": True}},
    },
}
BASELINE_PUBLISHED = None  # the reference publishes no throughput number


def layout_of(workload: str, n_gpus: int) -> dict:
    w = WORKLOADS[workload]
    if n_gpus not in w["layouts"]:
        raise SystemExit(f"--config {workload} runs on {sorted(w['layouts'])} GPUs, "
                         f"not {n_gpus}")
    lay = {"tensor": 1, "pipeline": 1, "context": 1, "data": 1, "virtual": 1}
    lay.update(w["layouts"][n_gpus])
    return lay


def layout_name(lay: dict) -> str:
    parts = [f"{n}{lay[k]}" for n, k in (("tp", "tensor"), ("cp", "context"),
                                          ("pp", "pipeline"), ("dp", "data")) if lay[k] > 1]
    if lay["virtual"] > 1:
        parts.append(f"v{lay['virtual']}")
    return "".join(parts) or "tp1"


def micro_batch_of(workload: str, n_gpus: int, override: int | None = None) -> int:
    """Micro-batch size: ``override`` if given, else the workload's value for this GPU
    count (an int, or a mapping GPU count -> int). The global batch never changes."""
    if override:
        return int(override)
    mb = WORKLOADS[workload]["micro_batch"]
    return int(mb[n_gpus]) if isinstance(mb, dict) else int(mb)


def make_config_dict(n_gpus: int, steps: int, workload: str = "311m", *,
                     reference: bool = False, micro_batch: int | None = None) -> dict:
    w = WORKLOADS[workload]
    lay = layout_of(workload, n_gpus)
    tp, pp, dp = lay["tensor"], lay["pipeline"], lay["data"]
    mb = micro_batch_of(workload, n_gpus, micro_batch)
    if w["global_batch"] % (mb * dp):
        raise SystemExit(f"global batch {w['global_batch']} is not a multiple of micro-batch "
                         f"{mb} x DP {dp}")
    gas = w["global_batch"] // (mb * dp)
    horizon = max(10488, steps + 100)
    d = {
        "distributed": {"backend": "nccl", "device": "cuda", "timeout_minutes": 5},
        "parallel": {"tensor": tp, "pipeline": pp, "context": lay["context"], "expert": 1,
                     "data": dp, "order": ["tp", "cp", "ep", "dp", "pp"],
                     "sequence_parallel": tp > 1},
        "model": dict(w["model"]),
        "precision": {"params": "bfloat16", "compute": "bfloat16", "grad_reduce": "float32"},
        "data_parallel": {"mode": "ddp", "bucket_bytes": 268435456, "overlap_grad_reduce": True},
        "pipeline": {"schedule": "1f1b", "overlap_p2p": True},
        "optimizer": {"lr": 3e-4, "betas": [0.9, 0.95], "eps": 1e-8, "weight_decay": 0.1,
                      "clip_grad_norm": 1.0},
        "lr_scheduler": {"schedule": "cosine", "warmup_steps": 0, "decay_steps": horizon,
                         "min_lr": 3e-5},
        "training": {"micro_batch_size": mb, "gradient_accumulation_steps": gas,
                     "max_steps": horizon, "seed": 1234, "log_interval": 10},
    }
    sections = dict(w.get("sections", {}))
    if reference:
        sections.update(w.get("reference_sections", {}))
    for k, v in sections.items():
        d.setdefault(k, {}).update(v)
    if lay["virtual"] > 1:
        d["pipeline"].update(schedule="interleaved_1f1b", virtual_stages_per_rank=lay["virtual"])
    return d


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks, power and clock-event reasons of one GPU during the timed region.

    Reads NVML in-process (read-only queries) every ``interval_s``; when NVML is not
    importable it runs ``nvidia-smi`` instead. The GPU is addressed by UUID, so the sample
    comes from the device this rank computes on even when CUDA_VISIBLE_DEVICES renumbers
    devices."""

    REASON_BITS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
                   "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
                   "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
                   "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str, *, interval_s: float = 0.2, nvml=None) -> None:
        self.uuid = device_uuid if device_uuid.startswith("GPU-") else f"GPU-{device_uuid}"
        self.interval_s = interval_s
        self.samples: list[tuple[float, float, set]] = []   # (sm MHz, max MHz, reasons)
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._read = self._nvml_reader(nvml) or self._smi_read

    @classmethod
    def for_device(cls, device) -> "ClockSampler":
        import torch

        return cls(str(torch.cuda.get_device_properties(device).uuid))

    def _nvml_reader(self, nvml):
        try:
            if nvml is None:
                import pynvml as nvml
            nvml.nvmlInit()
            h = nvml.nvmlDeviceGetHandleByUUID(self.uuid)
        except Exception:  # noqa: BLE001 - no NVML: fall back to nvidia-smi
            return None
        bits = {name: getattr(nvml, attr) for name, attr in self.REASON_BITS.items()}

        def read():
            sm = float(nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM))
            mx = float(nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM))
            mask = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(h))
            return sm, mx, {n for n, b in bits.items() if mask & b}
        return read

    def _smi_read(self):
        out = subprocess.run(["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.QUERY}",
                              "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5).stdout
        r = [c.strip() for c in out.strip().splitlines()[0].split(",")]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        return float(r[1]), float(r[2]), {n for n, v in zip(names, r[5:9])
                                          if v.lower() == "active"}

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.samples.append(self._read())
            except Exception:  # noqa: BLE001 - a failed sample is skipped
                pass
            self._stop.wait(self.interval_s)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        sm = sorted(x[0] for x in self.samples)
        reasons = set().union(*(x[2] for x in self.samples)) if self.samples else set()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": max(x[1] for x in self.samples) if self.samples else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


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

    d = make_config_dict(args.gpus, args.steps + args.warmup, args.config,
                         micro_batch=args.micro_batch)
    d["kernels"] = {"backend": "b200", "fused_tp_comm": not args.no_fused_tp,
                    "cuda_graphs": not args.no_cuda_graphs}
    cfg = config_from_dict(d)
    runtime = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, runtime)
    device = runtime.device
    trainer = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                      data_parallel=comps.data_parallel, rng=comps.rng, device=device)
    w = WORKLOADS[args.config]
    rows = w["global_batch"] // comps.parallel.dp.size
    batches = synthetic_batches(4, rows, w["model"]["seq_length"], w["model"]["vocab_size"],
                                seed=1234 + comps.parallel.coordinate.dp)
    src = trainer.batch_router.is_source
    lib = _ext.lib()
    try:
        with ClockSampler.for_device(device) as clocks:
            dev_ms, _, launches = run_timed(trainer, batches, args.steps, args.warmup, device,
                                            src, e2e=False, lib=lib)
        e2e_ms, e2e_wall, _ = run_timed(trainer, batches, args.steps, 0, device, src, e2e=True)
        _ext.check_status(device)
        report(args, rank, dev_ms, e2e_ms, e2e_wall, clocks.summary(), launches, impl="ours")
        if args.breakdown:
            kernel_breakdown(trainer, batches, device, src, args.breakdown, rank)
    finally:
        # graphs (holding NCCL work) -> TP barrier -> unmap peers -> barrier -> free own
        # buffer -> subgroups -> default group; see distributed/shutdown.py
        comps.close(trainer)
    return 0


def kernel_breakdown(trainer, batches, device, is_source, out_dir: str, rank: int) -> None:
    """Diagnostic, after the timed steps: one more train step under ``torch.profiler``;
    writes this rank's device time per kernel name (sorted, with shares of the step's
    kernel time) to ``out_dir/kernels_rank<r>.json``. Profiler times are for shares only,
    never for the reported throughput."""
    import torch

    os.makedirs(out_dir, exist_ok=True)
    barrier_sync(device)
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        trainer.train_step(batches[0] if is_source else None)
        torch.cuda.synchronize(device)
    totals: dict = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            t = totals.setdefault(ev.name, [0.0, 0])
            t[0] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time
            t[1] += 1
    rows = sorted(((n, us, c) for n, (us, c) in totals.items()), key=lambda r: -r[1])
    total = sum(r[1] for r in rows) or 1.0
    out = {"rank": rank, "kernel_us_total": total,
           "kernels": [{"name": n[:160], "us": round(us, 1), "launches": c,
                        "share": round(us / total, 4)} for n, us, c in rows]}
    with open(os.path.join(out_dir, f"kernels_rank{rank}.json"), "w") as f:
        json.dump(out, f, indent=1)
    barrier_sync(device)


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

    d = make_config_dict(args.gpus, args.steps + args.warmup, args.config, reference=True,
                         micro_batch=args.micro_batch)
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
    if cfg.pipeline.virtual_stages_per_rank > 1:
        built = builder.build_pipeline(cfg.model, parallel, kernels,
                                       virtual_stages_per_rank=cfg.pipeline.virtual_stages_per_rank,
                                       rng=rng)
    else:
        built = builder.build_stage(cfg.model, parallel, kernels, rng=rng)
    dtype = {"bfloat16": torch.bfloat16, "float32": torch.float32}[cfg.precision.params.value]
    model = built.model.to(device=runtime.device, dtype=dtype)
    strategy = build_data_parallel_strategy(cfg.data_parallel, cfg.offload, parallel,
                                            built.parameter_domains)
    trainer = Trainer(config=cfg, model=model, parallel=parallel, data_parallel=strategy,
                      rng=rng)
    device = runtime.device
    w = WORKLOADS[args.config]
    rows = w["global_batch"] // parallel.dp.size
    batches = synthetic_batches(4, rows, w["model"]["seq_length"], w["model"]["vocab_size"],
                                seed=1234 + parallel.coordinate.dp)
    src = trainer.batch_router.is_source
    try:
        with ClockSampler.for_device(device) as clocks:
            dev_ms, _, _ = run_timed(trainer, batches, args.steps, args.warmup, device, src,
                                     e2e=False)
        e2e_ms, e2e_wall, _ = run_timed(trainer, batches, args.steps, 0, device, src, e2e=True)
        report(args, rank, dev_ms, e2e_ms, e2e_wall, clocks.summary(), None, impl="reference")
    finally:
        import torch.distributed as dist

        torch.cuda.synchronize(device)
        del trainer
        if dist.is_available() and dist.is_initialized():
            dist.barrier(device_ids=[device.index])
        parallel.close()
        runtime.close()
    return 0


def unavailable(why: str) -> int:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
    return 0


def model_flops_per_token(m: dict) -> float:
    """Training FLOPs per token of the GPT (forward + backward = 3 x forward): 6 x the
    parameters of every matrix product (QKV, output, gate/up, down, LM head) plus causal
    attention, 6 x layers x hidden x sequence (score and value products over half the
    context on average). Recomputation under activation checkpointing is not counted."""
    h, f, layers = m["hidden_size"], m["ffn_hidden_size"], m["layers"]
    hq = m["heads"]
    hkv = m.get("kv_heads") or hq
    d = h // hq
    per_layer = h * (hq + 2 * hkv) * d + h * h + h * 2 * f + f * h
    return 6.0 * (layers * per_layer + m["vocab_size"] * h) + 6.0 * layers * h * m["seq_length"]


def roofline(w: dict, tokens_per_s: float, n_gpus: int) -> dict:
    """Model TFLOP/s per GPU and its fraction of the measured sustained bf16 GEMM rate
    (``MEASURED_PEAKS.json``, when present)."""
    per_gpu = model_flops_per_token(w["model"]) * tokens_per_s / n_gpus / 1e12
    out = {"model_flops_per_token": model_flops_per_token(w["model"]),
           "model_tflops_per_gpu": per_gpu}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            sustained = json.load(fh).get("bf16_tflops_sustained")
        if sustained:
            out["frac_of_measured_bf16_sustained"] = per_gpu / float(sustained)
    return out


def report(args, rank, dev_ms, e2e_ms, e2e_wall_ms, clocks, launches, *, impl):
    w = WORKLOADS[args.config]
    seq, gb = w["model"]["seq_length"], w["global_batch"]
    tokens_per_step = gb * seq
    value = tokens_per_step * args.steps / (dev_ms / 1000.0)
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)
    lay = layout_of(args.config, args.gpus)
    line = {
        "metric": METRIC.format(w["title"]),
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None if BASELINE_PUBLISHED is None else value / BASELINE_PUBLISHED,
        "dtype": "bf16", "data": "synthetic uniform-random token ids, random-init weights",
        "config": {"model": w["describe"], "name": args.config,
                   "global_batch": gb, "seq_len": seq,
                   "micro_batch": micro_batch_of(args.config, args.gpus, args.micro_batch),
                   "parallelism": layout_name(lay),
                   "l2": "no flush: weights (>= 622 MB) and activations exceed the 126 MB L2"},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "wall_ms_per_step": e2e_wall_ms / args.steps,
                "h2d_bytes_per_step": 2 * (gb // lay["data"]) * seq * 8,
                "d2h_bytes_per_step": 8},
        "impl": impl,
    }
    if launches is not None:
        line["gpu_launches"] = launches
    try:
        line["roofline"] = roofline(w, value, args.gpus)
    except Exception as error:  # noqa: BLE001 - an annotation never costs the measurement
        line["roofline"] = {"error": repr(error)}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1, choices=[1, 2, 4, 8])
    ap.add_argument("--config", default="311m", choices=sorted(WORKLOADS),
                    help="benchmark workload (default: the headline 311M config)")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-fused-tp", action="store_true",
                    help="diagnostic: NCCL all-gather/reduce-scatter instead of the fused "
                         "NVLink AG->GEMM / GEMM->RS kernels")
    ap.add_argument("--no-cuda-graphs", action="store_true",
                    help="diagnostic: launch every kernel from Python instead of replaying one "
                         "CUDA graph per microbatch")
    ap.add_argument("--micro-batch", type=int, default=None,
                    help="override the workload's micro-batch size (global batch unchanged)")
    ap.add_argument("--breakdown", default=None, metavar="DIR",
                    help="diagnostic: after timing, profile one more step and write per-kernel "
                         "device times per rank to DIR")
    args = ap.parse_args()
    rank, world, local = dist_env()
    layout_of(args.config, args.gpus)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    if args.impl == "reference":
        return run_reference(args, rank, world, local)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
