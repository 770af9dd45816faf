"""Sequence sharding for context parallelism (contiguous or zigzag)."""

from __future__ import annotations

import torch


def chunk_ids(rank: int, size: int, load_balance: bool) -> tuple[int, ...]:
    """Global chunk indices held by ``rank`` (chunks of S/CP, or S/(2CP) when balanced)."""
    return (rank, 2 * size - 1 - rank) if load_balance else (rank,)


def local_positions(seq_local: int, rank: int, size: int, load_balance: bool = False
                    ) -> torch.Tensor:
    if not load_balance:
        return torch.arange(rank * seq_local, (rank + 1) * seq_local)
    c = seq_local // 2
    a, b = chunk_ids(rank, size, True)
    return torch.cat([torch.arange(a * c, (a + 1) * c), torch.arange(b * c, (b + 1) * c)])


def shard_sequence(t: torch.Tensor, rank: int, size: int, *, load_balance: bool = False,
                   dim: int = 1) -> torch.Tensor:
    """This rank's part of a full-sequence tensor (sequence along ``dim``)."""
    if size == 1:
        return t
    n = t.shape[dim]
    if not load_balance:
        if n % size:
            raise ValueError(f"sequence length {n} is not divisible by CP size {size}")
        s = n // size
        return t.narrow(dim, rank * s, s)
    if n % (2 * size):
        raise ValueError(f"sequence length {n} is not divisible by 2*CP ({2 * size})")
    c = n // (2 * size)
    a, b = chunk_ids(rank, size, True)
    return torch.cat([t.narrow(dim, a * c, c), t.narrow(dim, b * c, c)], dim)


def unshard_sequence(parts: list[torch.Tensor], *, load_balance: bool = False, dim: int = 1
                     ) -> torch.Tensor:
    """Inverse of :func:`shard_sequence` given every rank's part in rank order."""
    size = len(parts)
    if not load_balance:
        return torch.cat(parts, dim)
    c = parts[0].shape[dim] // 2
    chunks = [None] * (2 * size)
    for r, p in enumerate(parts):
        a, b = chunk_ids(r, size, True)
        chunks[a] = p.narrow(dim, 0, c)
        chunks[b] = p.narrow(dim, c, c)
    return torch.cat(chunks, dim)


def gathered_to_global_order(size: int, load_balance: bool) -> list[tuple[int, int]]:
    """For each global chunk, the (rank, half) holding it in a rank-major gather."""
    if not load_balance:
        return [(r, 0) for r in range(size)]
    out = []
    for c in range(2 * size):
        out.append((c, 0) if c < size else (2 * size - 1 - c, 1))
    return out
