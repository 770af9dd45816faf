"""Checkpoint save / resume with the reference's directory layout.

``<run dir>/step_%08d/`` holds (src/nano_megatron/checkpoint/manager.py:105-1280):

* ``manifest.json`` (schema 2) and a ``.complete`` marker written last;
* single process: ``model.pt`` (backend ``torch.save``) + ``data_parallel.pt``;
* several ranks: ``rank_states/tpXXXX_ppXXXX_epXXXX.pt`` = ``{"model", "data_parallel"}``
  written by the dp = cp = 0 rank of each (tp, pp, ep) coordinate (backend
  ``rank_local_torch.save``; every data-parallel mode, ZeRO-3 included, since the
  strategies here gather their state to logical, DP-size-independent tensors);
* ``rank_runtime/tpXXXX_ppXXXX_cpXXXX_epXXXX_dpXXXX.pt`` per rank (torch CPU/CUDA
  RNG + ParallelRNG counters) and ``trainer_state.pt``.

Failures are collective: a write error on any rank is gathered and raised on
every rank (and stays raised for an async save). Files are written to a
temporary name and renamed; retention keeps ``keep_last`` complete checkpoints
plus the pinned best-validation one. Async saves snapshot to host memory,
write from one background thread, and publish manifest + ``.complete`` in
``flush()``.
"""

from __future__ import annotations

import contextlib
import copy
import dataclasses
import json
import math
import os
import shutil
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping

import torch
import torch.distributed as dist

from .manifest import (
    CheckpointManifest,
    RankLocalShard,
    RankRuntimeState,
    make_manifest,
    validate_topology,
)
from .fsdp2_format import (SHARD_INFO_FILE, from_fsdp2_state, load_dcp, load_dcp_model,
                           save_dcp, to_fsdp2_state, zero3_state_dir)
from .mapping import ShardedState

BEST_VALIDATION_FILE = "best_validation.json"
BEST_VALIDATION_VERSION = 1


def _dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def _world() -> int:
    return dist.get_world_size() if _dist() else 1


def _rank() -> int:
    return dist.get_rank() if _dist() else 0


def _barrier() -> None:
    if _dist():
        if dist.get_backend() == "nccl" and torch.cuda.is_available():
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def _all_gather_object(obj) -> list:
    if not _dist():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def _atomic_write_bytes(path: Path, writer) -> None:
    tmp = path.with_name(f".{path.name}.tmp")
    writer(tmp)
    os.replace(tmp, path)


def _torch_save(obj, path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    _atomic_write_bytes(path, lambda p: torch.save(obj, p))


def _atomic_text(path: Path, text: str) -> None:
    _atomic_write_bytes(path, lambda p: p.write_text(text))


def _torch_load(path: Path):
    return torch.load(path, map_location="cpu", weights_only=False)


def capture_runtime_state(rng) -> dict[str, Any]:
    state: dict[str, Any] = {"torch_cpu_rng": torch.get_rng_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["torch_cuda_rng"] = torch.cuda.get_rng_state(torch.cuda.current_device())
    if rng is not None:
        state["explicit_rng"] = copy.deepcopy(rng.state_dict())
    return state


def restore_runtime_state(state: Mapping[str, Any], rng) -> None:
    cpu = state.get("torch_cpu_rng")
    if not isinstance(cpu, torch.Tensor):
        raise ValueError("rank runtime state is missing torch CPU RNG")
    cuda = state.get("torch_cuda_rng")
    if cuda is not None and not torch.cuda.is_available():
        raise RuntimeError("checkpoint contains CUDA RNG state but CUDA is unavailable")
    explicit = state.get("explicit_rng")
    if explicit is not None and rng is None:
        raise ValueError("checkpoint contains explicit RNG state but no RNG object was passed")
    torch.set_rng_state(cpu)
    if cuda is not None:
        torch.cuda.set_rng_state(cuda, torch.cuda.current_device())
    if explicit is not None:
        rng.load_state_dict(explicit)


def _canonical(model):
    return getattr(model, "module", model)


def _virtual_stages(model) -> int:
    chunks = getattr(_canonical(model), "chunks", None)
    return len(chunks) if chunks is not None else 1


@dataclass
class _Pending:
    target: Path
    future: Future | None
    manifest_args: dict


class CheckpointManager:
    def __init__(self, *, config, parallel, run_config=None) -> None:
        self.config = config
        self.parallel = parallel
        self.run_config = run_config
        self.directory = Path(getattr(config, "directory", "checkpoints"))
        self.keep_last = int(getattr(config, "keep_last", 2))
        if self.keep_last < 0:
            raise ValueError("checkpoint.keep_last cannot be negative")
        self.async_save = bool(getattr(config, "async_save", False))
        self._executor = ThreadPoolExecutor(max_workers=1, thread_name_prefix="nmb-checkpoint") \
            if self.async_save else None
        self._pending: _Pending | None = None
        self._async_error: BaseException | None = None
        self._closed = False

    # ------------------------------------------------------------------ errors
    def _collective_error(self, local: BaseException | None, *, message: str) -> None:
        errs = _all_gather_object(None if local is None else repr(local))
        bad = [(r, e) for r, e in enumerate(errs) if e is not None]
        if bad:
            detail = "; ".join(f"rank {r}: {e}" for r, e in bad)
            raise RuntimeError(f"{message}: {detail}") from local

    def _preflight(self, target: Path) -> None:
        err = None
        if _rank() == 0:
            try:
                if target.exists() and not (target / ".complete").is_file() and any(target.iterdir()):
                    raise FileExistsError(f"incomplete checkpoint directory already exists: "
                                          f"{target}")
                if (target / ".complete").is_file():
                    raise FileExistsError(f"checkpoint already exists: {target}")
                target.mkdir(parents=True, exist_ok=True)
            except BaseException as e:  # noqa: BLE001
                err = e
        self._collective_error(err, message=f"checkpoint preflight failed for {target}")

    # ------------------------------------------------------------------ save
    def save(self, step: int, *, model, data_parallel, trainer_state: Mapping[str, Any],
             path: Path | str | None = None, rng=None) -> Path:
        if self._closed:
            raise RuntimeError("checkpoint manager is closed")
        if self._async_error is not None:
            raise RuntimeError("a previous asynchronous checkpoint failed") from self._async_error
        if step < 0:
            raise ValueError("checkpoint step cannot be negative")
        self.flush()
        target = Path(path) if path is not None else self.directory / f"step_{step:08d}"
        self._preflight(target)
        runtime = capture_runtime_state(rng)
        mode = str(getattr(data_parallel, "mode", "unknown"))
        registry = getattr(data_parallel, "parameter_domains", None)
        canon = _canonical(model)
        dtype = _param_dtype(self.run_config)
        full = getattr(data_parallel, "full_parameters", None)
        with full() if callable(full) else contextlib.nullcontext():
            sharded = ShardedState.from_model(canon, parameter_domains=registry,
                                              parallel=self.parallel, dtype=dtype)
        dp_state = data_parallel.state_dict()
        payloads: list[tuple[Any, Path]] = []
        c = self.parallel.coordinate
        if mode == "zero3":
            # The reference's ZeRO-3 layout: one DCP directory per (tp, pp) coordinate with
            # the model and a per-parameter AdamW state; plus our shard description (layer
            # ranges, TP shard metadata) for export.
            backend = "fsdp2_dcp"
            metadata, local_shard = {}, None
            if c.dp == 0 and c.cp == 0:
                b1, b2, eps, wd = data_parallel._opt_hparams()
                nested = to_fsdp2_state(sharded.state, dp_state, data_parallel.buffers.buckets,
                                        betas=(b1, b2), eps=eps, weight_decay=wd)
                d = zero3_state_dir(target, c.tp, c.pp)
                info = dataclasses.replace(self._local_shard(canon, sharded),
                                           state_file=str(d.relative_to(target)))
                payloads.append((_DCPPayload(nested), d))
                payloads.append((_JSONPayload(info.to_dict()), d / SHARD_INFO_FILE))
        elif _world() == 1:
            backend = "torch.save"
            payloads.append((sharded.state, target / "model.pt"))
            payloads.append((dict(dp_state), target / "data_parallel.pt"))
            metadata, local_shard = sharded.metadata, None
        else:
            backend = "rank_local_torch.save"
            metadata = {}
            local_shard = None
            if c.dp == 0 and c.cp == 0:
                local_shard = self._local_shard(canon, sharded)
                payloads.append(({"model": sharded.state, "data_parallel": dict(dp_state)},
                                 target / local_shard.state_file))
        rt = self._runtime_entry()
        payloads.append((runtime, target / rt.state_file))
        if _rank() == 0:
            payloads.append((dict(trainer_state), target / "trainer_state.pt"))
        shards = self._gather_shards(local_shard) if backend == "rank_local_torch.save" else ()
        runtimes = self._gather_runtime(rt)
        args = dict(step=step, storage_backend=backend, metadata=metadata, data_parallel_mode=mode,
                    rank_local_shards=shards, rank_runtime_states=runtimes,
                    virtual_stages_per_rank=_virtual_stages(model))
        if self._executor is not None:
            fut = self._executor.submit(_write_payloads, payloads)
            self._pending = _Pending(target, fut, args)
            return target
        err = None
        try:
            _write_payloads(payloads)
        except BaseException as e:  # noqa: BLE001
            err = e
        self._collective_error(err, message=f"checkpoint write failed for {target}")
        self._publish(target, args)
        return target

    def _local_shard(self, model, sharded: ShardedState) -> RankLocalShard:
        c = self.parallel.coordinate
        sid = f"tp{c.tp:04d}_pp{c.pp:04d}_ep{c.ep:04d}"
        part = getattr(model, "partition", None)
        if part is not None:
            ranges = ((int(part.start_layer), int(part.end_layer)),)
        else:
            ranges = tuple((int(ch.partition.start_layer), int(ch.partition.end_layer))
                           for ch in getattr(model, "chunks", ()) if hasattr(ch, "partition"))
        return RankLocalShard(sid, int(self.parallel.rank), c.tp, c.pp, c.ep, c.cp, c.dp,
                              f"rank_states/{sid}.pt", dict(sharded.metadata),
                              None if part is None else int(part.start_layer),
                              None if part is None else int(part.end_layer), ranges)

    def _runtime_entry(self) -> RankRuntimeState:
        c = self.parallel.coordinate
        sid = f"tp{c.tp:04d}_pp{c.pp:04d}_cp{c.cp:04d}_ep{c.ep:04d}_dp{c.dp:04d}"
        return RankRuntimeState(sid, int(self.parallel.rank), c.tp, c.pp, c.cp, c.ep, c.dp,
                                f"rank_runtime/{sid}.pt")

    def _gather_shards(self, local: RankLocalShard | None) -> tuple:
        got = [s for s in _all_gather_object(local) if s is not None]
        shards = tuple(sorted(got, key=lambda s: (s.pp, s.tp, s.ep)))
        want = self.parallel.tp.size * self.parallel.pp.size * self.parallel.ep.size
        if len(shards) != want:
            raise RuntimeError(f"collected {len(shards)} rank-local checkpoint shards, expected "
                               f"{want}")
        return shards

    def _gather_runtime(self, local: RankRuntimeState) -> tuple:
        return tuple(sorted(_all_gather_object(local), key=lambda s: s.writer_rank))

    def _publish(self, target: Path, args: dict) -> None:
        err = None
        if _rank() == 0:
            try:
                m = make_manifest(parallel=self.parallel,
                                  run_config=portable_run_config(self.run_config), **args)
                _atomic_text(target / "manifest.json",
                             json.dumps(m.to_dict(), indent=2, sort_keys=True) + "\n")
                _atomic_text(target / ".complete", "complete\n")
                if target.parent.resolve() == self.directory.resolve():
                    self._remove_old(exclude=target)
            except BaseException as e:  # noqa: BLE001
                err = e
        self._collective_error(err, message=f"checkpoint publish failed for {target}")
        _barrier()

    def flush(self) -> None:
        """Wait for an asynchronous save and publish it (collective)."""
        pending, self._pending = self._pending, None
        if pending is None:
            return
        err = None
        try:
            if pending.future is not None:
                pending.future.result()
        except BaseException as e:  # noqa: BLE001
            err = e
        try:
            self._collective_error(err, message=f"asynchronous checkpoint failed for "
                                                f"{pending.target}")
        except BaseException as e:
            self._async_error = e
            raise
        self._publish(pending.target, pending.manifest_args)

    def close(self) -> None:
        if self._closed:
            return
        try:
            self.flush()
        finally:
            if self._executor is not None:
                self._executor.shutdown(wait=True)
            self._closed = True

    def __enter__(self) -> "CheckpointManager":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # ------------------------------------------------------------------ load
    def load(self, path: Path | str, *, model, data_parallel, rng=None) -> dict[str, Any]:
        self.flush()
        path = Path(path)
        if not (path / ".complete").is_file():
            raise FileNotFoundError(f"checkpoint is incomplete or missing: {path}")
        manifest = CheckpointManifest.read(path / "manifest.json")
        validate_topology(manifest, self.parallel)
        canon = _canonical(model)
        mode = str(getattr(data_parallel, "mode", "unknown"))
        if manifest.data_parallel_mode not in ("unknown", mode):
            raise ValueError(f"checkpoint data-parallel mode {manifest.data_parallel_mode!r} "
                             f"does not match {mode!r}")
        if manifest.storage_backend == "rank_local_torch.save":
            shard = self._select_shard(manifest)
            rel = Path(shard.state_file)
            if rel.is_absolute() or ".." in rel.parts:
                raise ValueError(f"invalid rank-local state path in manifest: {shard.state_file}")
            payload = _torch_load(path / rel)
            model_state, dp_state = payload.get("model"), payload.get("data_parallel")
        elif manifest.storage_backend == "torch.save":
            model_state = _torch_load(path / "model.pt")
            dp_state = _torch_load(path / "data_parallel.pt")
        elif manifest.storage_backend == "fsdp2_dcp":
            c = self.parallel.coordinate
            nested = load_dcp(zero3_state_dir(path, c.tp, c.pp))
            model_state = nested["model"]
            dp_state = from_fsdp2_state(nested, data_parallel.buffers.buckets, mode=mode)
        elif manifest.storage_backend == "torch.distributed.checkpoint":
            # single-process checkpoints written by the reference (DCP directory "dcp/")
            model_state = load_dcp_model(path / "dcp")
            dp_state = _torch_load(path / "data_parallel.pt")
        else:
            raise ValueError(f"unsupported checkpoint backend {manifest.storage_backend!r}")
        if not isinstance(model_state, Mapping) or not isinstance(dp_state, Mapping):
            raise ValueError("checkpoint is missing model or data-parallel state")
        full = getattr(data_parallel, "full_parameters", None)
        with torch.no_grad(), (full() if callable(full) else contextlib.nullcontext()):
            canon.load_state_dict(dict(model_state))
        data_parallel.load_state_dict(dict(dp_state))
        self._load_runtime(path, manifest, rng)
        state = _torch_load(path / "trainer_state.pt")
        if not isinstance(state, Mapping):
            raise ValueError("trainer_state.pt does not contain a mapping")
        return {"trainer_state": dict(state), "manifest": manifest}

    def _select_shard(self, manifest: CheckpointManifest) -> RankLocalShard:
        c = self.parallel.coordinate
        cands = [s for s in manifest.rank_local_shards if s.tp == c.tp and s.pp == c.pp]
        exact = [s for s in cands if s.ep == c.ep]
        if exact:
            return exact[0]
        expert = any(m.parameter_domain.value == "expert" for s in cands
                     for m in s.tensor_metadata.values())
        if cands and not expert:
            return min(cands, key=lambda s: s.ep)
        raise ValueError(f"checkpoint has no rank-local shard for coordinate tp={c.tp}, "
                         f"pp={c.pp}, ep={c.ep}")

    def _load_runtime(self, path: Path, manifest: CheckpointManifest, rng) -> None:
        c = self.parallel.coordinate
        match = [s for s in manifest.rank_runtime_states
                 if (s.tp, s.pp, s.cp, s.ep, s.dp) == (c.tp, c.pp, c.cp, c.ep, c.dp)]
        if not match:
            import warnings

            warnings.warn("no saved runtime RNG state for this coordinate (new data-parallel "
                          "replica); keeping the freshly initialised RNG state", stacklevel=2)
            return
        restore_runtime_state(_torch_load(path / match[0].state_file), rng)

    # ------------------------------------------------------------------ discovery
    def latest(self) -> Path | None:
        if not self.directory.exists():
            return None
        done = sorted(p for p in self.directory.glob("step_*")
                      if p.is_dir() and (p / ".complete").is_file())
        return done[-1] if done else None

    def best_validation(self) -> dict[str, Any] | None:
        path = self.directory / BEST_VALIDATION_FILE
        if not path.exists():
            return None
        v = json.loads(path.read_text())
        if set(v) != {"checkpoint", "format_version", "metric", "mode", "step", "value"}:
            raise ValueError("best-validation checkpoint pin has invalid fields")
        if v["format_version"] != BEST_VALIDATION_VERSION or v["metric"] != "loss" or \
                v["mode"] != "min":
            raise ValueError("best-validation checkpoint pin metric contract is invalid")
        if v["checkpoint"] != f"step_{int(v['step']):08d}":
            raise ValueError("best-validation checkpoint pin path does not match its step")
        if not (self.directory / v["checkpoint"] / ".complete").is_file():
            raise ValueError("best-validation checkpoint pin points to an incomplete checkpoint")
        return dict(v)

    def pin_best_validation(self, step: int, loss: float) -> Path:
        if isinstance(step, bool) or not isinstance(step, int) or step < 0:
            raise ValueError("best-validation step must be a non-negative integer")
        if not math.isfinite(float(loss)) or float(loss) < 0:
            raise ValueError("best-validation loss must be finite and non-negative")
        self.flush()
        target = self.directory / f"step_{step:08d}"
        err = None
        if _rank() == 0:
            try:
                if not (target / ".complete").is_file():
                    raise ValueError(f"cannot pin incomplete best-validation checkpoint: {target}")
                _atomic_text(self.directory / BEST_VALIDATION_FILE, json.dumps(
                    {"checkpoint": target.name, "format_version": BEST_VALIDATION_VERSION,
                     "metric": "loss", "mode": "min", "step": step, "value": float(loss)},
                    indent=2, sort_keys=True) + "\n")
                self._remove_old(exclude=target)
            except BaseException as e:  # noqa: BLE001
                err = e
        self._collective_error(err, message=f"best-validation checkpoint pin failed for {target}")
        return target

    def _remove_old(self, *, exclude: Path) -> None:
        pinned = None
        try:
            pinned = (self.best_validation() or {}).get("checkpoint")
        except ValueError:
            pinned = None
        done = sorted(p for p in self.directory.glob("step_*")
                      if p.is_dir() and (p / ".complete").is_file())
        keep = set(done[-self.keep_last:]) if self.keep_last else set()
        for p in done:
            if p in keep or p.resolve() == exclude.resolve() or p.name == pinned:
                continue
            shutil.rmtree(p, ignore_errors=True)


# Config fields this framework adds to the reference's schema, with their defaults.
# They are left out of the manifest's run_config while at the default, so that the
# reference's own config loader (which rejects unknown fields) can read the manifest.
_EXTENSION_FIELDS = {("kernels", "cuda_graphs"): True, ("kernels", "fused_tp_comm"): True,
                     ("kernels", "fused_dp_comm"): True, ("kernels", "fused_cp_comm"): True,
                     ("kernels", "deterministic"): False,
                     ("context_parallel", "load_balance"): False}


def portable_run_config(run_config):
    from .manifest import json_compatible

    if run_config is None:
        return None
    d = json_compatible(run_config)
    if not isinstance(d, dict):
        return d
    for (section, name), default in _EXTENSION_FIELDS.items():
        sec = d.get(section)
        if isinstance(sec, dict) and sec.get(name, default) == default:
            sec.pop(name, None)
    # kernels.backend "b200" names this framework's kernel set; the reference's schema
    # knows only "torch", its own default kernels, which is what a reader should use.
    if isinstance(d.get("kernels"), dict) and d["kernels"].get("backend") == "b200":
        d["kernels"]["backend"] = "torch"
    return d


@dataclass
class _DCPPayload:
    """A nested state written as a single-writer torch.distributed.checkpoint directory."""
    state: dict


@dataclass
class _JSONPayload:
    value: Any


def _write_payloads(payloads) -> None:
    for obj, path in payloads:
        if isinstance(obj, _DCPPayload):
            save_dcp(obj.state, path)
        elif isinstance(obj, _JSONPayload):
            path.parent.mkdir(parents=True, exist_ok=True)
            path.write_text(json.dumps(obj.value, indent=1, sort_keys=True))
        else:
            _torch_save(obj, path)


def _param_dtype(run_config) -> torch.dtype | None:
    prec = getattr(run_config, "precision", None)
    name = str(getattr(getattr(prec, "params", None), "value", getattr(prec, "params", "")))
    return {"float32": torch.float32, "bfloat16": torch.bfloat16,
            "float16": torch.float16}.get(name)
