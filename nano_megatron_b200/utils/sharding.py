"""Map full (TP=1) model weights to tensor-parallel shards and back.

A parameter's shard dimension comes from its layer type: column-parallel
weights (and biases) and the vocab-parallel embedding / LM head split dim 0,
row-parallel weights split dim 1, everything else is replicated. Used by the
checkpoint export (merge) and by tests that compare a TP layout with a
single-rank model.
"""

from __future__ import annotations

import re

import torch

_DIM0 = re.compile(r"(q_proj|k_proj|v_proj|gate_proj|up_proj)\.linear\.(weight|bias)$"
                   r"|embedding\.weight$|lm_head\.(weight|bias)$")
_DIM1 = re.compile(r"(out_proj|down_proj)\.linear\.weight$")


def tensor_shard_dim(name: str) -> int | None:
    if _DIM1.search(name):
        return 1
    if _DIM0.search(name):
        return 0
    return None


def shard_tensor(t: torch.Tensor, dim: int | None, rank: int, size: int) -> torch.Tensor:
    if dim is None or size == 1:
        return t
    n = t.shape[dim] // size
    return t.narrow(dim, rank * n, n)


def pad_vocab(t: torch.Tensor, padded: int) -> torch.Tensor:
    if t.shape[0] >= padded:
        return t
    pad = torch.zeros((padded - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype)
    return torch.cat([t, pad], 0)


def shard_state_dict(full: dict, rank: int, size: int) -> dict:
    return {k: shard_tensor(v, tensor_shard_dim(k), rank, size).clone() for k, v in full.items()}


def merge_shards(shards: list[dict]) -> dict:
    out = {}
    for k in shards[0]:
        d = tensor_shard_dim(k)
        out[k] = shards[0][k] if d is None or len(shards) == 1 else \
            torch.cat([s[k] for s in shards], d)
    return out
