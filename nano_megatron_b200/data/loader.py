"""Deterministic, exactly resumable batch loading over the (DP, EP) batch replicas.

Sample order is the one ``torch.utils.data.DistributedSampler`` defines
(per-epoch ``randperm`` seeded ``seed + epoch`` when shuffling, truncated to a
multiple of the replica count, replica ``r`` taking every ``R``-th index from
``r``), so a given seed visits the same samples as the reference's loader
(src/nano_megatron/data/loader.py:41-315). Progress is one global sample
offset inside the current epoch, advanced only when a complete batch is
handed to the trainer; it is topology-explicit, so a data-parallel reshard
resumes the same global prefix.

Batches of token-stream datasets are gathered by the native prefetcher: the
window indices of the next ``prefetch`` batches are queued to a C++ worker that
copies them (widening uint16/uint32 to int64) straight into fresh pinned host
buffers, which the trainer then copies to the GPU asynchronously.
"""

from __future__ import annotations

import atexit
import hashlib
import json
import weakref
from collections import deque
from collections.abc import Iterator, Mapping
from typing import Any

import torch
from torch.utils.data import DistributedSampler

from .datasets import RandomTokenDataset, build_train_dataset


def _nonneg(name: str, v) -> int:
    if isinstance(v, bool) or not isinstance(v, int):
        raise TypeError(f"{name} must be an integer")
    if v < 0:
        raise ValueError(f"{name} must be non-negative")
    return v


class _Sized:
    def __init__(self, n: int) -> None:
        self.n = n

    def __len__(self) -> int:
        return self.n


def epoch_indices(n: int, *, replicas: int, rank: int, shuffle: bool, seed: int,
                  epoch: int) -> list[int]:
    """The replica's sample order for one epoch (drop-last distributed sampling)."""
    s = DistributedSampler(_Sized(n), num_replicas=replicas, rank=rank, shuffle=shuffle,
                           seed=seed, drop_last=True)
    s.set_epoch(epoch)
    return list(iter(s))


_LIVE: "weakref.WeakSet[StatefulDataLoader]" = weakref.WeakSet()


@atexit.register
def _close_live_loaders() -> None:
    for ld in list(_LIVE):
        try:
            ld.close()
        except Exception:  # noqa: BLE001
            pass


class StatefulDataLoader(Iterator):
    STATE_VERSION = 1

    def __init__(self, dataset, *, local_batch_size: int, replica_count: int, replica_index: int,
                 shuffle: bool, shuffle_seed: int, data_fingerprint: str,
                 pin_memory: bool = False, prefetch: int = 2, threads: int = 4) -> None:
        self.dataset = dataset
        self.local_batch_size = int(local_batch_size)
        self.replica_count = int(replica_count)
        self.replica_index = int(replica_index)
        self.shuffle = bool(shuffle)
        self.shuffle_seed = _nonneg("shuffle_seed", shuffle_seed)
        self.data_fingerprint = data_fingerprint
        self.pin_memory = bool(pin_memory)
        self.prefetch = max(1, int(prefetch))
        self.threads = int(threads)
        self.epoch = 0
        self.sample_offset = 0
        n = len(dataset)
        per_replica = n // self.replica_count
        self.samples_per_epoch = (per_replica // self.local_batch_size) * \
            self.local_batch_size * self.replica_count
        self.global_batch_size = self.local_batch_size * self.replica_count
        if self.samples_per_epoch < self.global_batch_size:
            raise ValueError("training dataset does not provide one complete global batch")
        self._order: list[int] | None = None
        self._cursor = 0           # next local index position to *submit*
        self._queue: deque = deque()
        self._prefetcher = None
        self._native = hasattr(dataset, "native_source") and hasattr(dataset, "window_starts")
        _LIVE.add(self)

    # ------------------------------------------------------------------ properties
    epoch_seed = property(lambda self: self.shuffle_seed + self.epoch)
    batches_per_epoch = property(lambda self: self.samples_per_epoch // self.global_batch_size)
    num_workers = property(lambda self: 0)

    def __len__(self) -> int:
        return self.batches_per_epoch

    def __iter__(self) -> "StatefulDataLoader":
        return self

    # ------------------------------------------------------------------ batches
    def _start_epoch(self) -> None:
        if self.sample_offset % self.replica_count:
            raise RuntimeError("global data sample_offset cannot be divided across current "
                               f"replicas: {self.sample_offset} % {self.replica_count} != 0")
        self._drop_queue()
        self._order = epoch_indices(len(self.dataset), replicas=self.replica_count,
                                    rank=self.replica_index, shuffle=self.shuffle,
                                    seed=self.shuffle_seed, epoch=self.epoch)
        self._cursor = self.sample_offset // self.replica_count

    def _local_epoch_end(self) -> int:
        return self.samples_per_epoch // self.replica_count

    def _buffer(self) -> torch.Tensor:
        w = self.dataset.sequence_length + 1
        return torch.empty(self.local_batch_size, w, dtype=torch.int64,
                           pin_memory=self.pin_memory)

    def _submit_one(self) -> bool:
        if self._cursor + self.local_batch_size > self._local_epoch_end():
            return False
        idx = self._order[self._cursor:self._cursor + self.local_batch_size]
        self._cursor += self.local_batch_size
        if self._native:
            if self._prefetcher is None:
                from nano_megatron_b200.native import native

                self._prefetcher = native().BatchPrefetcher(self.dataset.native_source(),
                                                            self.dataset.sequence_length + 1,
                                                            self.threads)
            out = self._buffer()
            starts = self.dataset.window_starts(torch.tensor(idx, dtype=torch.int64))
            self._queue.append((self._prefetcher.submit(starts.contiguous(), out), out))
        else:
            self._queue.append((None, idx))
        return True

    def _fill(self) -> None:
        while len(self._queue) < self.prefetch and self._submit_one():
            pass

    def _drop_queue(self) -> None:
        while self._queue:
            job, out = self._queue.popleft()
            if job is not None:
                self._prefetcher.wait(job)

    def _materialise(self, job, payload) -> dict[str, torch.Tensor]:
        if job is not None:
            self._prefetcher.wait(job)
            buf = payload
        else:
            ds = self.dataset
            rows = [ds.window(i) if isinstance(ds, RandomTokenDataset)
                    else torch.cat([ds[i]["input_ids"], ds[i]["labels"][-1:]]) for i in payload]
            buf = torch.stack(rows)
            if self.pin_memory:
                buf = buf.pin_memory()
        return {"input_ids": buf[:, :-1], "labels": buf[:, 1:]}

    def __next__(self) -> dict[str, torch.Tensor]:
        if self._order is None:
            self._start_epoch()
        self._fill()
        if not self._queue:
            raise RuntimeError("stateful data loader ended before its committed epoch boundary: "
                               f"offset={self.sample_offset}, "
                               f"epoch_samples={self.samples_per_epoch}")
        job, payload = self._queue.popleft()
        batch = self._materialise(job, payload)
        self.sample_offset += self.global_batch_size
        if self.sample_offset > self.samples_per_epoch:
            raise RuntimeError("stateful data loader advanced beyond the epoch boundary")
        if self.sample_offset == self.samples_per_epoch:
            self.epoch += 1
            self.sample_offset = 0
            self._order = None
        else:
            self._fill()
        return batch

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, int]:
        return {"version": self.STATE_VERSION, "epoch": self.epoch,
                "shuffle_seed": self.shuffle_seed, "epoch_seed": self.epoch_seed,
                "sample_offset": self.sample_offset, "samples_per_epoch": self.samples_per_epoch}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        ver = int(state.get("version", self.STATE_VERSION))
        if ver != self.STATE_VERSION:
            raise ValueError(f"unsupported stateful DataLoader state version: {ver}")
        epoch = _nonneg("data epoch", int(state.get("epoch", 0)))
        seed = state.get("shuffle_seed", state.get("seed"))
        seed = self.shuffle_seed if seed is None else _nonneg("data shuffle_seed", int(seed))
        if seed != self.shuffle_seed:
            raise RuntimeError(f"training shuffle seed changed across resume: {seed} != "
                               f"{self.shuffle_seed}")
        es = int(state.get("epoch_seed", seed + epoch))
        if es != seed + epoch:
            raise ValueError(f"data epoch_seed is inconsistent with shuffle_seed + epoch: {es} "
                             f"!= {seed + epoch}")
        spe = state.get("samples_per_epoch")
        if spe is not None and int(spe) != self.samples_per_epoch:
            raise RuntimeError("samples per epoch changed across resume; exact data restoration "
                               f"is impossible: {spe} != {self.samples_per_epoch}")
        off = _nonneg("data sample_offset", int(state.get("sample_offset", 0)))
        self._check_offset(off)
        self._drop_queue()
        self.epoch, self.sample_offset, self._order = epoch, off, None

    def seek_consumed_samples(self, consumed: int) -> None:
        consumed = _nonneg("consumed_samples", consumed)
        if consumed % self.global_batch_size:
            raise RuntimeError("restored consumed_samples is incompatible with the current global "
                               f"batch size: {consumed} % {self.global_batch_size} != 0")
        self._drop_queue()
        self.epoch, self.sample_offset = divmod(consumed, self.samples_per_epoch)
        self._check_offset(self.sample_offset)
        self._order = None

    def _check_offset(self, off: int) -> None:
        if off >= self.samples_per_epoch and off != 0:
            raise ValueError(f"data sample_offset must be inside the current epoch: {off} >= "
                             f"{self.samples_per_epoch}")
        if off % self.global_batch_size:
            raise RuntimeError("data sample_offset is incompatible with the current global batch "
                               f"size: {off} % {self.global_batch_size} != 0")

    def close(self) -> None:
        self._drop_queue()
        if self._prefetcher is not None:
            self._prefetcher.shutdown()
            self._prefetcher = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


def _local_batch(config) -> int:
    return int(config.training.micro_batch_size) * int(config.training.gradient_accumulation_steps)


def _target(config, max_steps) -> int:
    t = config.training.max_steps if max_steps is None else max_steps
    if isinstance(t, bool) or not isinstance(t, int):
        raise TypeError("max_steps must be an integer")
    if t < 1:
        raise ValueError("max_steps must be positive")
    return t


def _capacity(ds, replicas: int, local: int) -> None:
    if len(ds) // replicas < local:
        raise ValueError("training dataset is too short for one complete epoch batch after "
                         f"sharding: got {len(ds)} samples for {replicas} DP×EP replicas and "
                         f"local_batch_size={local}; need at least {replicas * local} samples")


def _pin(parallel) -> bool:
    rt = getattr(parallel, "runtime", None)
    dev = getattr(rt, "device_type", None) or getattr(getattr(rt, "device", None), "type", None)
    return dev == "cuda" and torch.cuda.is_available()


def build_train_dataloader(config, parallel, tokenizer=None, *, max_steps: int | None = None,
                           start_step: int = 0, consumed_samples: int = 0):
    """Infinite, exactly resumable loader on each batch-replica source rank (others: empty)."""
    steps = _target(config, max_steps)
    start = _nonneg("start_step", start_step)
    consumed = _nonneg("consumed_samples", consumed_samples)
    if parallel.batch_replica.rank != 0:
        return iter(())
    replicas = int(parallel.topology.batch_replica_size)
    local = _local_batch(config)
    ds = build_train_dataset(config, tokenizer)
    need = steps * local * replicas
    if isinstance(ds, RandomTokenDataset) and len(ds) < need:
        ds = RandomTokenDataset(num_samples=need, sequence_length=config.model.seq_length,
                                vocab_size=config.model.vocab_size, seed=config.training.seed)
    _capacity(ds, replicas, local)
    fp = getattr(ds, "fingerprint", None)
    if not isinstance(fp, str) or not fp:
        raise TypeError("training dataset must expose a non-empty fingerprint")
    data_fp = hashlib.sha256(json.dumps(
        {"dataset": fp, "sampler": "stateful-torch-distributed-sampler-v2",
         "seed": int(config.training.seed), "shuffle": bool(config.data.shuffle)},
        sort_keys=True, separators=(",", ":")).encode("utf-8")).hexdigest()
    c = parallel.coordinate
    loader = StatefulDataLoader(ds, local_batch_size=local, replica_count=replicas,
                                replica_index=c.dp * parallel.topology.expert_parallel_size + c.ep,
                                shuffle=bool(config.data.shuffle),
                                shuffle_seed=int(config.training.seed), data_fingerprint=data_fp,
                                pin_memory=_pin(parallel))
    if consumed:
        loader.seek_consumed_samples(consumed)
    elif start:
        loader.seek_consumed_samples(start * loader.global_batch_size)
    return loader


class ValidationLoader:
    """Finite, unshuffled replica shard of the validation data (re-iterable)."""

    def __init__(self, dataset, *, local_batch_size: int, replica_count: int, replica_index: int,
                 seed: int, pin_memory: bool) -> None:
        self.dataset = dataset
        self.local = local_batch_size
        self.order = epoch_indices(len(dataset), replicas=replica_count, rank=replica_index,
                                   shuffle=False, seed=seed, epoch=0)
        self.pin_memory = pin_memory

    def __len__(self) -> int:
        return len(self.order) // self.local

    def __iter__(self):
        ds = self.dataset
        for b in range(len(self)):
            idx = self.order[b * self.local:(b + 1) * self.local]
            if hasattr(ds, "native_source"):
                buf = torch.empty(self.local, ds.sequence_length + 1, dtype=torch.int64,
                                  pin_memory=self.pin_memory)
                ds.native_source().gather(ds.window_starts(torch.tensor(idx)), buf.shape[1], buf,
                                          4)
            else:
                buf = torch.stack([torch.cat([ds[i]["input_ids"], ds[i]["labels"][-1:]])
                                   for i in idx])
            yield {"input_ids": buf[:, :-1], "labels": buf[:, 1:]}


def build_validation_dataloader(config, parallel, tokenizer=None):
    v = config.validation
    if int(v.interval) <= 0:
        return iter(())
    if v.data is None:
        raise ValueError("validation.interval > 0 requires validation.data")
    if parallel.batch_replica.rank != 0:
        return iter(())
    replicas = int(parallel.topology.batch_replica_size)
    local = _local_batch(config)
    ds = build_train_dataset(config, tokenizer, data_config=v.data)
    _capacity(ds, replicas, local)
    c = parallel.coordinate
    loader = ValidationLoader(ds, local_batch_size=local, replica_count=replicas,
                              replica_index=c.dp * parallel.topology.expert_parallel_size + c.ep,
                              seed=int(config.training.seed), pin_memory=_pin(parallel))
    if len(loader) < int(v.batches):
        raise ValueError("validation dataset is too short for validation.batches complete global "
                         f"batches: got {len(ds)} samples, need at least "
                         f"{int(v.batches) * local * replicas}")
    return loader
