"""Deterministic, checkpointable RNG streams derived from parallel coordinates.

The seed derivation is part of the reference's observable behaviour (initial
weights and dropout masks depend on it), so it is reproduced exactly:
``blake2b("base|stream|coords...|components...", digest 8 B, person
b"nano-mgt")`` little-endian ``% (2**63 - 1)``, with DATA keyed by (dp, ep),
DENSE_INIT by (tp, pp), EXPERT_INIT by (tp, pp, ep), ACTIVATION by (dp, ep)
(src/nano_megatron/parallel/rng.py:25-186).
"""

from __future__ import annotations

import hashlib
import threading
from collections.abc import Iterator, Mapping, Sequence
from contextlib import contextmanager
from enum import StrEnum
from typing import Any

from .axes import ParallelCoordinate


class RNGStream(StrEnum):
    DATA = "data"
    DENSE_INIT = "dense_init"
    EXPERT_INIT = "expert_init"
    ACTIVATION = "activation"


_KEY_AXES = {
    RNGStream.DATA: ("dp", "ep"),
    RNGStream.DENSE_INIT: ("tp", "pp"),
    RNGStream.EXPERT_INIT: ("tp", "pp", "ep"),
    RNGStream.ACTIVATION: ("dp", "ep"),
}


class ParallelRNG:
    MAX_SEED = 2**63 - 1

    def __init__(self, base_seed: int, coordinate: ParallelCoordinate) -> None:
        if isinstance(base_seed, bool) or not isinstance(base_seed, int) or base_seed < 0:
            raise ValueError("base_seed must be a non-negative integer")
        if not isinstance(coordinate, ParallelCoordinate):
            raise TypeError("coordinate must be a ParallelCoordinate")
        self.base_seed = base_seed
        self.coordinate = coordinate
        self._counters = dict.fromkeys(RNGStream, 0)
        self._lock = threading.Lock()

    @classmethod
    def from_context(cls, base_seed: int, parallel) -> "ParallelRNG":
        return cls(base_seed, parallel.coordinate)

    def seed(self, stream: RNGStream | str, *components: int | str) -> int:
        s = RNGStream(stream)
        coords = [f"{a}={getattr(self.coordinate, a)}" for a in _KEY_AXES[s]]
        text = "|".join([str(self.base_seed), s.value, *coords, *map(str, components)])
        digest = hashlib.blake2b(text.encode(), digest_size=8, person=b"nano-mgt").digest()
        return int.from_bytes(digest, "little") % self.MAX_SEED

    def next_seed(self, stream: RNGStream | str, *components: int | str) -> int:
        s = RNGStream(stream)
        with self._lock:
            n = self._counters[s]
            self._counters[s] = n + 1
        return self.seed(s, n, *components)

    def activation_seed(self, *, layer: int, microbatch: int, global_token_offset: int = 0,
                        op: str = "dropout") -> int:
        for name, v in (("layer", layer), ("microbatch", microbatch),
                        ("global_token_offset", global_token_offset)):
            if isinstance(v, bool) or not isinstance(v, int) or v < 0:
                raise ValueError(f"{name} must be a non-negative integer")
        return self.seed(RNGStream.ACTIVATION, layer, microbatch, global_token_offset, op)

    def generator(self, stream: RNGStream | str, *, device: str = "cpu",
                  components: Sequence[int | str] = (), advance: bool = True):
        import torch

        seed = self.next_seed(stream, *components) if advance else self.seed(stream, *components)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        return gen

    @contextmanager
    def fork(self, stream: RNGStream | str, *, components: Sequence[int | str] = (),
             cuda_devices: Sequence[int] | None = None, advance: bool = True) -> Iterator[int]:
        """Seed torch's default CPU (and listed CUDA) generators inside the block only."""
        import torch

        seed = self.next_seed(stream, *components) if advance else self.seed(stream, *components)
        devices = list(cuda_devices or ())
        with torch.random.fork_rng(devices=devices, enabled=True):
            torch.random.default_generator.manual_seed(seed)
            for d in devices:
                with torch.cuda.device(d):
                    torch.cuda.manual_seed(seed)
            yield seed

    def state_dict(self) -> dict[str, Any]:
        with self._lock:
            counters = {s.value: n for s, n in self._counters.items()}
        c = self.coordinate
        return {"base_seed": self.base_seed,
                "coordinate": {"tp": c.tp, "cp": c.cp, "ep": c.ep, "dp": c.dp, "pp": c.pp},
                "counters": counters}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        if state.get("base_seed") != self.base_seed:
            raise ValueError(f"RNG base seed mismatch: state has {state.get('base_seed')}, "
                             f"expected {self.base_seed}")
        mine = self.state_dict()["coordinate"]
        if state.get("coordinate") != mine:
            raise ValueError(f"RNG coordinate mismatch: state has {state.get('coordinate')}, "
                             f"expected {mine}")
        counters = state.get("counters")
        if not isinstance(counters, Mapping):
            raise ValueError("RNG state must contain a counters mapping")
        parsed = {}
        for s in RNGStream:
            v = counters.get(s.value)
            if isinstance(v, bool) or not isinstance(v, int) or v < 0:
                raise ValueError(f"invalid counter for RNG stream {s.value!r}: {v!r}")
            parsed[s] = v
        with self._lock:
            self._counters.update(parsed)
