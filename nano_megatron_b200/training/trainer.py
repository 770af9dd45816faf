"""Training loop: train_step / evaluate / fit with device-side metrics.

Behaviour of the reference Trainer (src/nano_megatron/training/trainer.py:
117-894): the step routes the batch (source rank -> batch-replica peers, CP
slicing), splits microbatches, zeroes grads, runs the pipeline schedule,
synchronises tied embeddings, finalises the data-parallel reduction, clips,
steps the optimizer and the LR schedule, and aggregates token-weighted loss
metrics. Differences, B200-first: the step never synchronises with the host
(loss sums, token counts and the gradient norm stay on the device until a log
interval), it is timed with CUDA events (max over ranks), and checkpoint /
validation / metric-history hooks run between steps.
"""

from __future__ import annotations

import math
import time
from pathlib import Path
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from nano_megatron_b200.utils.profiling import nvtx_range
from nano_megatron_b200.utils.timing import DeviceStepTimer, StepPhaseTimer, summarize_phases

from .batch_router import BatchRouter
from .lr_scheduler import LearningRateScheduler
from .metrics import aggregate_loss_metrics
from .microbatches import split_microbatches


@dataclass
class TrainerState:
    step: int = 0
    consumed_samples: int = 0
    consumed_tokens: int = 0
    data_fingerprint: str | None = None
    data_epoch: int = 0
    data_shuffle_seed: int | None = None
    data_sample_offset: int = 0
    data_samples_per_epoch: int | None = None
    lr_scheduler: dict | None = None
    wandb_run_id: str | None = None
    metrics_history: dict | None = None
    best_validation_loss: float | None = None
    best_validation_step: int | None = None
    best_validation_checkpoint: str | None = None

    _FIELDS = ("step", "consumed_samples", "consumed_tokens", "data_fingerprint", "data_epoch",
               "data_shuffle_seed", "data_sample_offset", "data_samples_per_epoch",
               "lr_scheduler", "wandb_run_id", "metrics_history", "best_validation_loss",
               "best_validation_step", "best_validation_checkpoint")

    def state_dict(self) -> dict[str, Any]:
        out = {k: getattr(self, k) for k in self._FIELDS}
        for k in ("lr_scheduler", "metrics_history"):
            if out[k] is not None:
                out[k] = dict(out[k])
        return out

    def load_state_dict(self, state: dict[str, Any]) -> None:
        for k in ("step", "consumed_samples", "consumed_tokens", "data_epoch",
                  "data_sample_offset"):
            v = int(state.get(k, 0))
            if v < 0:
                raise ValueError(f"trainer {k} must be non-negative")
            setattr(self, k, v)
        seed = state.get("data_shuffle_seed")
        if seed is not None and int(seed) < 0:
            raise ValueError("trainer data_shuffle_seed must be non-negative or null")
        self.data_shuffle_seed = None if seed is None else int(seed)
        spe = state.get("data_samples_per_epoch")
        if spe is not None and int(spe) < 1:
            raise ValueError("trainer data_samples_per_epoch must be positive or null")
        self.data_samples_per_epoch = None if spe is None else int(spe)
        fp = state.get("data_fingerprint")
        if fp is not None and (not isinstance(fp, str) or not fp):
            raise ValueError("trainer data_fingerprint must be a non-empty string or null")
        self.data_fingerprint = fp
        sched = state.get("lr_scheduler")
        if sched is not None and not isinstance(sched, dict):
            raise ValueError("trainer lr_scheduler state must be a mapping or null")
        self.lr_scheduler = None if sched is None else dict(sched)
        rid = state.get("wandb_run_id")
        if rid is not None and (not isinstance(rid, str) or not rid):
            raise ValueError("trainer wandb_run_id must be a non-empty string or null")
        self.wandb_run_id = rid
        mh = state.get("metrics_history")
        if mh is not None and not isinstance(mh, dict):
            raise ValueError("trainer metrics_history state must be a mapping or null")
        self.metrics_history = None if mh is None else dict(mh)
        bl, bs, bc = (state.get("best_validation_loss"), state.get("best_validation_step"),
                      state.get("best_validation_checkpoint"))
        if bl is None and bs is None:
            if bc is not None:
                raise ValueError("trainer best_validation_checkpoint requires best validation "
                                 "metrics")
            self.best_validation_loss = self.best_validation_step = None
            self.best_validation_checkpoint = None
            return
        if isinstance(bl, bool) or not isinstance(bl, (int, float)) or not math.isfinite(bl) \
                or bl < 0:
            raise ValueError("trainer best_validation_loss must be finite and non-negative")
        if isinstance(bs, bool) or not isinstance(bs, int) or bs < 0:
            raise ValueError("trainer best_validation_step must be a non-negative integer")
        self.best_validation_loss, self.best_validation_step = float(bl), bs
        self.best_validation_checkpoint = bc


def check_token_ranges(batch, vocab_size: int) -> None:
    """Reject a batch whose token ids fall outside the vocabulary, on the host.

    The fused kernels treat an id outside a rank's vocabulary shard as "another rank's
    token" (a zero embedding row, no logit of its own), which is right for shards but
    would silently train on garbage for an id outside the whole vocabulary, e.g. after a
    tokenizer/model mismatch. Inputs must lie in [0, vocab_size); labels below 0 are
    ignored positions and otherwise must lie below vocab_size. Only CPU tensors are checked
    (before the copy to the device), so the check never synchronises with the GPU.
    """
    if not isinstance(batch, dict):
        return
    for key, allow_negative in (("input_ids", False), ("labels", True)):
        t = batch.get(key)
        if not isinstance(t, torch.Tensor) or t.is_cuda or t.numel() == 0:
            continue
        hi, lo = int(t.max()), int(t.min())
        if hi >= vocab_size or (lo < 0 and not allow_negative):
            bad = hi if hi >= vocab_size else lo
            raise ValueError(f"batch[{key!r}] holds token id {bad}, outside the model's "
                             f"vocabulary of {vocab_size} (model.vocab_size)")


def _move_to_device(batch, device):
    if isinstance(batch, torch.Tensor):
        return batch.to(device, non_blocking=True)
    if isinstance(batch, dict):
        return {k: _move_to_device(v, device) for k, v in batch.items()}
    return batch


class Trainer:
    def __init__(self, *, config, model, parallel, data_parallel, checkpoint=None,
                 data_iterator=None, metrics_path=None, resume_metrics_path=None, rng=None,
                 device=None, health=None) -> None:
        self.config = config
        self.model = model
        self.parallel = parallel
        self.data_parallel = data_parallel
        self.checkpoint = checkpoint
        self.data_iterator = data_iterator
        self.rng = rng
        self.health = health            # PeerHealth: host-side failure detection, optional
        self.profiler = None            # utils.profiling.StepProfiler, optional
        self.state = TrainerState()
        self.device = device or next(model.parameters()).device
        data_parallel.configure_precision(config.precision)
        configure_kernels = getattr(data_parallel, "configure_kernels", None)
        if callable(configure_kernels):
            configure_kernels(config.kernels)
        self.prepare_pipeline_stage()
        data_parallel.setup(model, config.optimizer, getattr(data_parallel, "parameter_domains",
                                                             None))
        self.batch_router = BatchRouter(parallel, load_balance=bool(
            getattr(config.context_parallel, "load_balance", False)))
        self.schedule = self._build_schedule()
        self.lr_scheduler = LearningRateScheduler(config=config.lr_scheduler,
                                                  optimizer_config=config.optimizer,
                                                  data_parallel=data_parallel,
                                                  max_steps=config.training.max_steps)
        self.timer = DeviceStepTimer(self.device)
        self.phases = StepPhaseTimer(self.device)
        self.last_step_ms: float | None = None
        self.metrics_path = metrics_path
        self.resume_metrics_path = resume_metrics_path
        from .wandb_logger import WandbLogger

        self.logger = WandbLogger(getattr(config, "wandb", None), run_config=config,
                                  is_primary=parallel.rank == 0,
                                  metrics_path=None if metrics_path is None else Path(metrics_path),
                                  resume_metrics_path=None if resume_metrics_path is None
                                  else Path(resume_metrics_path))
        self._restored_step: int | None = None
        self._restored_run_id: str | None = None
        self._restored_history = None
        self.validation_data = None
        self._hooks: list = []

    # ------------------------------------------------------------------ setup
    def prepare_pipeline_stage(self) -> None:
        sync = getattr(self.model, "synchronize_tied_embedding_weights", None)
        if callable(sync):
            sync()

    def _build_schedule(self):
        from nano_megatron_b200.pipeline_parallel.schedules import build_schedule

        return build_schedule(self.config, self.model, self.parallel, self.data_parallel)

    @property
    def micro_batch_size(self) -> int:
        return self.config.training.micro_batch_size

    # ------------------------------------------------------------------ steps
    def _prepare_batch(self, batch):
        check_token_ranges(batch, self.config.model.vocab_size)
        batch = self.batch_router.route(batch)
        batch = _move_to_device(batch, self.device)
        micro = split_microbatches(batch, self.micro_batch_size)
        out = []
        for i, mb in enumerate(micro):
            mb = dict(mb) if isinstance(mb, dict) else mb
            if isinstance(mb, dict):
                mb["_microbatch_index"] = i
            out.append(mb)
        return out

    def train_step(self, batch) -> dict[str, Any]:
        """One optimizer update. Returns device tensors (``loss``, ``grad_norm``...)."""
        with nvtx_range(f"step {self.state.step}"):
            return self._train_step(batch)

    def _train_step(self, batch) -> dict[str, Any]:
        self.model.train()
        micro = self._prepare_batch(batch)
        dp = self.data_parallel
        dp.zero_grad()
        acc = self.schedule.forward_backward(micro, forward_only=False)
        self.phases.mark("forward_backward")
        sync = getattr(self.model, "synchronize_tied_embedding_gradients", None)
        if callable(sync):
            sync()
        dp.finalize_gradients()
        self.phases.mark("grad_sync")
        clip = self.config.optimizer.clip_grad_norm
        grad_norm = dp.clip_grad_norm(clip)
        self.phases.mark("clip")
        lr_used = dp.learning_rate      # the rate this update applies (the one to log)
        dp.optimizer_step()
        self.phases.mark("optimizer")
        self.state.step += 1
        self.lr_scheduler.set_completed_steps(self.state.step)
        self.state.lr_scheduler = self.lr_scheduler.state_dict()
        gbs = self.config.training.micro_batch_size * \
            self.config.training.gradient_accumulation_steps * \
            self.parallel.dp.size * self.parallel.ep.size
        self.state.consumed_samples += gbs
        self.state.consumed_tokens += gbs * self.config.model.seq_length
        loss_sum, count = aggregate_loss_metrics(acc, self.parallel, self.device)
        return {"loss_sum": loss_sum, "token_count": count, "grad_norm": grad_norm,
                "learning_rate": lr_used}

    @torch.no_grad()
    def evaluate_step(self, batch) -> tuple[torch.Tensor, torch.Tensor]:
        self.model.eval()
        micro = self._prepare_batch(batch)
        acc = self.schedule.forward_backward(micro, forward_only=True)
        return aggregate_loss_metrics(acc, self.parallel, self.device)

    def evaluate(self, batches) -> dict[str, float]:
        total, count = 0.0, 0.0
        for b in batches:
            s, c = self.evaluate_step(b)
            total += float(s)
            count += float(c)
        loss = total / max(count, 1.0)
        return {"loss": loss, "perplexity": math.exp(min(loss, 50.0)), "token_count": count}

    def timed_train_step(self, batch) -> tuple[dict[str, Any], float]:
        """``train_step`` bracketed by CUDA events; returns (metrics, device ms)."""
        self.timer.start()
        out = self.train_step(batch)
        self.timer.stop()
        ms = self.timer.elapsed_ms()
        self.last_step_ms = ms
        return out, ms

    def bind_data_iterator(self, data, *, data_fingerprint: str | None = None) -> None:
        if self.state.data_fingerprint is not None and data_fingerprint is not None and \
                self.state.data_fingerprint != data_fingerprint:
            raise RuntimeError("data fingerprint changed across resume")
        self.state.data_fingerprint = data_fingerprint
        restore = getattr(data, "load_state_dict", None)
        if callable(restore) and self.state.step > 0:
            st = {"epoch": self.state.data_epoch, "sample_offset": self.state.data_sample_offset}
            if self.state.data_shuffle_seed is not None:
                st["shuffle_seed"] = self.state.data_shuffle_seed
            if self.state.data_samples_per_epoch is not None:
                st["samples_per_epoch"] = self.state.data_samples_per_epoch
            restore(st)
        self._data = data
        self.data_iterator = iter(data)

    def bind_validation_data(self, data) -> None:
        self.validation_data = data

    def _record_data_state(self) -> None:
        data = getattr(self, "_data", None)
        get = getattr(data, "state_dict", None)
        if callable(get):
            st = get()
            self.state.data_epoch = int(st.get("epoch", 0))
            self.state.data_shuffle_seed = st.get("shuffle_seed", st.get("seed"))
            self.state.data_sample_offset = int(st.get("sample_offset", 0))
            self.state.data_samples_per_epoch = st.get("samples_per_epoch")

    def start_logging(self) -> None:
        """Open the metric history (replaying a resumed checkpoint's prefix) and W&B."""
        rid = self.logger.start(checkpoint_run_id=self._restored_run_id,
                                checkpoint_step=self._restored_step,
                                checkpoint_metrics_state=self._restored_history, model=self.model)
        self.state.wandb_run_id = rid

    def fit(self, *, max_steps: int | None = None, log=print) -> TrainerState:
        """Train to ``max_steps``: log every ``log_interval`` steps, validate every
        ``validation.interval`` steps (saving and pinning an improved checkpoint), save every
        ``checkpoint.save_interval`` steps and once more at the end (``save_final``).
        Order of events per step follows the reference trainer
        (src/nano_megatron/training/trainer.py:580-700)."""
        self.start_logging()
        target = max_steps if max_steps is not None else self.config.training.max_steps
        interval = self.config.training.log_interval
        pending: list = []
        marks: list = []
        t0 = time.perf_counter()
        first_step = self.state.step
        self._last_saved = None
        health = getattr(self, "health", None)
        profiler = getattr(self, "profiler", None)
        while self.state.step < target:
            if health is not None:
                health.check()          # stop between steps if a peer failed
            if profiler is not None:
                profiler.before_step(self.state.step)
            data = getattr(self, "_data", None)
            saved = data.state_dict() if self.batch_router.is_source and \
                callable(getattr(data, "state_dict", None)) else None
            try:
                batch = next(self.data_iterator) if self.batch_router.is_source else None
                self.phases.begin()
                out = self.train_step(batch)
                step_marks = self.phases.end()
                if self.state.step % interval == 0 or self.state.step == target:
                    self._check_device_status()     # before logging, inside the failure path
            except BaseException as error:
                # Leave the data position at the last completed step (as the reference
                # does) so a checkpoint taken by the caller resumes exactly, and tell the
                # other ranks before they launch their next step.
                if saved is not None:
                    data.load_state_dict(saved)
                    self.data_iterator = iter(data)
                if health is not None:
                    health.report_failure(error)
                raise
            self._record_data_state()
            if profiler is not None:
                profiler.after_step(self.state.step)
            marks.append(step_marks)
            pending.append(out)
            if self.state.step % interval == 0 or self.state.step == target:
                self._log(pending, time.perf_counter() - t0, marks, log)
                pending, marks, t0 = [], [], time.perf_counter()
            self._after_step(log)
        ck = self.config.checkpoint
        if self.checkpoint is not None and ck.save_final and self.state.step > first_step and \
                self._last_saved != self.state.step:
            self.save_checkpoint()
        self.flush()
        return self.state

    def _after_step(self, log=print) -> None:
        for hook in self._hooks:
            hook(self)
        vc = self.config.validation
        if self.validation_data is not None and vc.interval and self.state.step % vc.interval == 0:
            self.run_validation(log)
        cp = self.checkpoint
        if cp is not None:
            iv = self.config.checkpoint.save_interval
            if iv and self.state.step % iv == 0 and \
                    getattr(self, "_last_saved", None) != self.state.step:
                self.save_checkpoint()

    def run_validation(self, log=print) -> dict[str, float]:
        """Evaluate ``validation.batches`` batches. Only batch-replica source ranks hold a
        validation loader; the others take part in every batch's routing and schedule with
        ``None``, so the source's batch count is shared with them first."""
        batches = []
        if self.batch_router.is_source:
            it = iter(self.validation_data)
            for _ in range(self.config.validation.batches):
                try:
                    batches.append(next(it))
                except StopIteration:
                    break
        g = self.batch_router.group
        if g is not None and g.size > 1:
            box = [len(batches) if self.batch_router.is_source else None]
            dist.broadcast_object_list(box, src=g.ranks[0], group=g.process_group)
            if not self.batch_router.is_source:
                batches = [None] * int(box[0])
        metrics = self.evaluate(batches)
        if self.parallel.rank == 0 and log is not None:
            log("validation " + " ".join(f"{k}={v:.6g}" for k, v in metrics.items()))
        self.logger.log("validation", metrics, state=self.state)
        best = self.state.best_validation_loss
        if best is None or metrics["loss"] < best:
            self.state.best_validation_loss = float(metrics["loss"])
            self.state.best_validation_step = self.state.step
            if self.checkpoint is not None and self.config.checkpoint.save_best_validation:
                self.state.best_validation_checkpoint = str(
                    Path(self.checkpoint.directory) / f"step_{self.state.step:08d}")
                path = self.save_checkpoint()
                pinned = self.checkpoint.pin_best_validation(self.state.step,
                                                             self.state.best_validation_loss)
                if Path(pinned) != Path(path):
                    raise RuntimeError("best-validation pin returned a different checkpoint "
                                       "path")
                self.logger.update_summary({"checkpoint/best_validation": str(path),
                                            "checkpoint/best_validation_loss":
                                                self.state.best_validation_loss,
                                            "checkpoint/best_validation_step": self.state.step})
        return metrics

    def _check_device_status(self) -> None:
        """Raise if one of this framework's kernels reported a bounded wait that ran out
        (the device status word; read at log time, when the host synchronises anyway)."""
        if self.device.type != "cuda":
            return
        from nano_megatron_b200.ops import _ext

        if _ext.available():
            _ext.check_status(self.device)

    def _log(self, pending, host_s, marks, log) -> None:
        """One log record for the steps in ``pending``. Device times come from the steps'
        phase marks (CUDA events), max over ranks per phase; ``time_<phase>_ms`` are
        per-step averages."""
        loss_sum = sum(float(p["loss_sum"]) for p in pending)
        count = sum(float(p["token_count"]) for p in pending)
        loss = loss_sum / max(count, 1.0)
        n = len(pending)
        # like the reference's metric store: the loss is token-weighted over the interval,
        # every other per-step metric (gradient norm, learning rate) is the interval mean
        gn = sum(float(p["grad_norm"]) for p in pending) / n
        lr = sum(float(p["learning_rate"]) for p in pending) / n
        gbs = self.config.training.micro_batch_size * \
            self.config.training.gradient_accumulation_steps * \
            self.parallel.dp.size * self.parallel.ep.size
        tokens = n * gbs * self.config.model.seq_length
        phases = summarize_phases(marks, self.device)
        dev_max = phases["step"]
        metrics = {"step": self.state.step, "loss": loss,
                   "perplexity": math.exp(min(loss, 50.0)), "token_count": count,
                   "grad_norm": gn, "learning_rate": lr,
                   "samples_per_second": n * gbs / max(host_s, 1e-9),
                   "tokens_per_second": tokens / max(host_s, 1e-9),
                   "tokens_per_second_device": tokens / max(dev_max / 1000.0, 1e-9)}
        for k, v in phases.items():
            metrics[f"time_{k}_ms"] = v / n
        self.last_step_ms = phases["step"] / n
        if self.device.type == "cuda":
            gib = 1024 ** 3
            metrics.update({
                "gpu_memory_allocated_gib": torch.cuda.memory_allocated(self.device) / gib,
                "gpu_memory_peak_allocated_gib": torch.cuda.max_memory_allocated(self.device) / gib,
                "gpu_memory_reserved_gib": torch.cuda.memory_reserved(self.device) / gib,
                "gpu_memory_peak_reserved_gib": torch.cuda.max_memory_reserved(self.device) / gib})
        self.last_metrics = metrics
        if self.parallel.rank == 0 and log is not None:
            log(" ".join(f"{k}={v:.6g}" if isinstance(v, float) else f"{k}={v}"
                         for k, v in metrics.items()))
        self.logger.log("train", {k: float(v) for k, v in metrics.items() if k != "step"},
                        state=self.state)

    # ------------------------------------------------------------------ checkpoints
    def save_checkpoint(self):
        if self.checkpoint is None:
            return None
        self.state.metrics_history = self.logger.history_state()
        path = self.checkpoint.save(step=self.state.step, model=self.model,
                                    data_parallel=self.data_parallel,
                                    trainer_state=self.state.state_dict(), rng=self.rng)
        self._last_saved = self.state.step
        self.logger.update_summary({"checkpoint/latest": str(path),
                                    "checkpoint/step": self.state.step})
        return path

    def load_checkpoint(self, path) -> None:
        loaded = self.checkpoint.load(path, model=self.model, data_parallel=self.data_parallel,
                                      rng=self.rng)
        self.state.load_state_dict(loaded["trainer_state"])
        self._restored_step = self.state.step
        self._restored_run_id = self.state.wandb_run_id
        self._restored_history = self.state.metrics_history
        if self.state.lr_scheduler is not None:
            self.lr_scheduler.load_state_dict(self.state.lr_scheduler,
                                              expected_completed_steps=self.state.step)
        else:
            self.lr_scheduler.set_completed_steps(self.state.step)

    def flush(self) -> None:
        if self.checkpoint is not None and hasattr(self.checkpoint, "flush"):
            self.checkpoint.flush()

    def release_graphs(self) -> None:
        """Drop every captured CUDA graph (and the device work handles of the data-parallel
        strategy). Graphs that captured NCCL collectives must be gone before the process
        groups are destroyed."""
        release = getattr(self.schedule, "release_graphs", None)
        if callable(release):
            release()
        drop = getattr(self.data_parallel, "release_pending_work", None)
        if callable(drop):
            drop()

    def close(self) -> None:
        try:
            self.flush()
        finally:
            self.logger.finish()
            close = getattr(getattr(self, "_data", None), "close", None)
            if callable(close):
                close()
