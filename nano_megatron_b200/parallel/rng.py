"""Named random streams whose seeds are a pure function of (base seed, stream, position).

Every random draw of a run (data order, weight init, dropout masks) comes from a named
stream. A stream's seed is a 64-bit hash of a short text key, so the same key gives the
same seed in every process, on every rank that shares the coordinates the stream is keyed
on, and after a restart. The key text, the hash (BLAKE2b, 8-byte digest, personalisation
``nano-mgt``, read little-endian, reduced mod 2**63 - 1) and the coordinates each stream
is keyed on are fixed by the reference's seeds (src/nano_megatron/parallel/rng.py:60-73,
173-186): weights and dropout masks are bit-identical across the two frameworks only if
they agree. Which coordinates key a stream decides what is shared:

==============  =============  =====================================================
stream          keyed on       consequence
==============  =============  =====================================================
data            dp, ep         each batch replica reads its own sample order
dense_init      tp, pp         TP shards differ, DP/CP/EP replicas start identical
expert_init     tp, pp, ep     expert weights also differ per EP rank
activation      dp, ep         dropout differs per batch replica, not per TP shard
==============  =============  =====================================================

Draws that must not repeat use a per-stream counter (``next_seed``); the counters are
the only mutable state, and they are what a checkpoint records.
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


STREAM_AXES: dict[RNGStream, tuple[str, ...]] = {
    RNGStream.DATA: ("dp", "ep"),
    RNGStream.DENSE_INIT: ("tp", "pp"),
    RNGStream.EXPERT_INIT: ("tp", "pp", "ep"),
    RNGStream.ACTIVATION: ("dp", "ep"),
}
_SEED_MODULUS = (1 << 63) - 1
_PERSON = b"nano-mgt"
_COORD_FIELDS = ("tp", "cp", "ep", "dp", "pp")


def stream_seed(base_seed: int, stream: RNGStream, coordinate: ParallelCoordinate,
                parts: Sequence[Any]) -> int:
    """Seed of ``stream`` at ``coordinate`` for the extra key ``parts``."""
    key = [str(base_seed), stream.value]
    key += [f"{axis}={getattr(coordinate, axis)}" for axis in STREAM_AXES[stream]]
    key += [str(p) for p in parts]
    h = hashlib.blake2b("|".join(key).encode("utf-8"), digest_size=8, person=_PERSON)
    return int.from_bytes(h.digest(), "little") % _SEED_MODULUS


def _is_count(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


class ParallelRNG:
    """The random streams of one rank (its parallel coordinate) for one base seed."""

    MAX_SEED = _SEED_MODULUS

    def __init__(self, base_seed: int, coordinate: ParallelCoordinate) -> None:
        if not _is_count(base_seed):
            raise ValueError(f"base seed must be an int >= 0, got {base_seed!r}")
        if not isinstance(coordinate, ParallelCoordinate):
            raise TypeError(f"expected a ParallelCoordinate, got {type(coordinate).__name__}")
        self.base_seed = base_seed
        self.coordinate = coordinate
        self._drawn = {s: 0 for s in RNGStream}      # draws taken from each stream so far
        self._mutex = threading.Lock()

    @classmethod
    def from_context(cls, base_seed: int, parallel) -> "ParallelRNG":
        return cls(base_seed, parallel.coordinate)

    # ------------------------------------------------------------------ seeds
    def seed(self, stream: RNGStream | str, *components: int | str) -> int:
        """Fixed seed of ``stream`` for the key ``components`` (no counter involved)."""
        return stream_seed(self.base_seed, RNGStream(stream), self.coordinate, components)

    def next_seed(self, stream: RNGStream | str, *components: int | str) -> int:
        """Seed of the stream's next draw: the draw index leads the key."""
        s = RNGStream(stream)
        with self._mutex:
            index = self._drawn[s]
            self._drawn[s] = index + 1
        return stream_seed(self.base_seed, s, self.coordinate, (index, *components))

    def activation_seed(self, *, layer: int, microbatch: int, global_token_offset: int = 0,
                        op: str = "dropout") -> int:
        """Seed of an activation op (dropout) at a (layer, microbatch, token offset): the
        same on every TP rank of a replica, so a mask never depends on the TP split."""
        key = {"layer": layer, "microbatch": microbatch,
               "global_token_offset": global_token_offset}
        bad = [k for k, v in key.items() if not _is_count(v)]
        if bad:
            raise ValueError("activation seed key must be ints >= 0: " +
                             ", ".join(f"{k}={key[k]!r}" for k in bad))
        return self.seed(RNGStream.ACTIVATION, layer, microbatch, global_token_offset, op)

    def _pick(self, stream, components, advance: bool) -> int:
        return self.next_seed(stream, *components) if advance else self.seed(stream, *components)

    # ------------------------------------------------------------------ torch generators
    def generator(self, stream: RNGStream | str, *, device: str = "cpu",
                  components: Sequence[int | str] = (), advance: bool = True):
        """A fresh ``torch.Generator`` on ``device`` seeded from the stream."""
        import torch

        g = torch.Generator(device=device)
        g.manual_seed(self._pick(stream, components, advance))
        return g

    @contextmanager
    def fork(self, stream: RNGStream | str, *, components: Sequence[int | str] = (),
             cuda_devices: Sequence[int] | None = None, advance: bool = True) -> Iterator[int]:
        """Run the block with torch's global CPU generator (and those of ``cuda_devices``)
        seeded from the stream; their previous states come back on exit."""
        import torch

        seed = self._pick(stream, components, advance)
        devices = list(cuda_devices or ())
        with torch.random.fork_rng(devices=devices, enabled=True):
            torch.random.default_generator.manual_seed(seed)
            for index in devices:
                with torch.cuda.device(index):
                    torch.cuda.manual_seed(seed)
            yield seed

    # ------------------------------------------------------------------ checkpoint
    def _coordinate_dict(self) -> dict[str, int]:
        return {axis: getattr(self.coordinate, axis) for axis in _COORD_FIELDS}

    def state_dict(self) -> dict[str, Any]:
        """``{"base_seed", "coordinate": {tp, cp, ep, dp, pp}, "counters": {stream: n}}``
        (the reference's checkpoint entry, so either framework resumes the other's)."""
        with self._mutex:
            drawn = {s.value: n for s, n in self._drawn.items()}
        return {"base_seed": self.base_seed, "coordinate": self._coordinate_dict(),
                "counters": drawn}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        """Restore the draw counters; the entry must come from the same seed and rank."""
        got_seed, got_coord = state.get("base_seed"), state.get("coordinate")
        if got_seed != self.base_seed:
            raise ValueError(f"checkpoint RNG entry was written for base seed {got_seed!r}, "
                             f"this run uses {self.base_seed}")
        if got_coord != self._coordinate_dict():
            raise ValueError(f"checkpoint RNG entry belongs to coordinate {got_coord!r}, "
                             f"this rank is {self._coordinate_dict()}")
        saved = state.get("counters")
        if not isinstance(saved, Mapping):
            raise ValueError("checkpoint RNG entry has no 'counters' mapping")
        restored = {s: saved.get(s.value) for s in RNGStream}
        broken = {s.value: v for s, v in restored.items() if not _is_count(v)}
        if broken:
            raise ValueError(f"checkpoint RNG counters must be ints >= 0: {broken}")
        with self._mutex:
            self._drawn.update(restored)
