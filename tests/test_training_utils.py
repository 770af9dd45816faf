"""Batch arithmetic, microbatch splitting and the context-parallel batch slice.

Mirrors the reference's training-utility unit tests (tests/unit/test_training_utils.py:30-97):
the global batch counts the expert axis as extra data replicas; nested batches split along
their leading dimension; inconsistent leading dimensions are rejected; every sequence
field (input ids, labels, positions, loss mask) is sliced to this context-parallel rank's
part, contiguously or zig-zag, and a sequence that does not divide is rejected.
"""

from __future__ import annotations

from collections import namedtuple
from dataclasses import dataclass

import pytest
import torch

from nano_megatron_b200.context_parallel.utils import unshard_sequence
from nano_megatron_b200.training.batch_router import shard_batch_for_context_parallel
from nano_megatron_b200.training.microbatches import global_batch_size, split_microbatches


def test_global_batch_includes_the_independent_expert_axis():
    assert global_batch_size(2, 3, 4, 1) == 24
    assert global_batch_size(2, 3, 4, 2) == 48
    with pytest.raises(ValueError):
        global_batch_size(0, 1, 1, 1)


Pair = namedtuple("Pair", "a b")


@dataclass
class Extra:
    mask: torch.Tensor
    tag: str


def test_split_nested_microbatches():
    batch = {"input_ids": torch.arange(12).view(6, 2),
             "nested": {"labels": torch.arange(6), "pair": Pair(torch.ones(6, 3), 7)},
             "extra": Extra(torch.zeros(6, 1), "x"),
             "scalar": torch.tensor(5.0)}
    parts = split_microbatches(batch, 2)
    assert len(parts) == 3
    p = parts[1]
    assert p["input_ids"].tolist() == [[4, 5], [6, 7]]
    assert p["nested"]["labels"].tolist() == [2, 3]
    assert p["nested"]["pair"].a.shape == (2, 3) and p["nested"]["pair"].b == 7
    assert p["extra"].mask.shape == (2, 1) and p["extra"].tag == "x"
    assert p["scalar"].item() == 5.0                  # 0-d tensors are shared, not split


def test_split_rejects_inconsistent_batch_dimensions():
    with pytest.raises(ValueError, match="leading dimension"):
        split_microbatches({"a": torch.zeros(4, 2), "b": torch.zeros(6, 2)}, 2)
    with pytest.raises(ValueError, match="not divisible"):
        split_microbatches({"a": torch.zeros(6, 2)}, 4)
    with pytest.raises(ValueError, match="no tensor"):
        split_microbatches({"a": 3}, 1)


def _batch(s=8):
    ids = torch.arange(2 * s).view(2, s)
    return {"input_ids": ids, "labels": ids + 100, "position_ids": ids % s,
            "loss_mask": (ids % 3 != 0).float(), "doc_id": torch.tensor([4, 9])}


@pytest.mark.parametrize("load_balance", [False, True], ids=["contiguous", "zigzag"])
def test_every_sequence_field_is_sliced_for_the_cp_rank(load_balance):
    b, size = _batch(), 2
    parts = [shard_batch_for_context_parallel(b, r, size, load_balance=load_balance)
             for r in range(size)]
    for k in ("input_ids", "labels", "position_ids", "loss_mask"):
        assert all(p[k].shape == (2, 4) for p in parts), k
        whole = unshard_sequence([p[k] for p in parts], load_balance=load_balance)
        assert torch.equal(whole, b[k]), k
    assert all(p["doc_id"] is b["doc_id"] for p in parts)      # not a sequence field
    if load_balance:   # rank 0 holds the first and the last quarter (causal work balance)
        assert parts[0]["input_ids"][0].tolist() == [0, 1, 6, 7]
    else:
        assert parts[1]["input_ids"][0].tolist() == [4, 5, 6, 7]


def test_cp_slice_rejects_a_sequence_that_does_not_divide():
    with pytest.raises(ValueError, match="not divisible by CP"):
        shard_batch_for_context_parallel(_batch(6), 0, 4)
    with pytest.raises(ValueError, match="2\\*CP"):
        shard_batch_for_context_parallel(_batch(6), 0, 2, load_balance=True)
    assert shard_batch_for_context_parallel(_batch(6), 0, 1) is not None


def test_interval_metrics_weight_loss_by_tokens_and_average_the_rest():
    """The reference's metric-store contract (tests/unit/test_metrics.py:30-54): the logged
    loss is sum(loss_sum) / sum(token_count) over the interval, perplexity its exponent,
    other metrics the interval mean; one process keeps the additive totals."""
    import math
    from types import SimpleNamespace

    from nano_megatron_b200.training.metrics import (MetricStore, aggregate_loss_metrics,
                                                     loss_and_perplexity)

    loss, ppl = loss_and_perplexity(4.0 + 9.0, 2.0 + 3.0)
    assert loss == pytest.approx(2.6) and ppl == pytest.approx(math.exp(2.6))
    assert loss_and_perplexity(1e4, 1.0)[1] == pytest.approx(math.exp(50.0))   # clamped
    store = MetricStore()
    for lr in (0.3, 0.1):
        store.add("lr", lr)
    assert store.mean("lr") == pytest.approx(0.2) and math.isnan(store.mean("absent"))
    store.clear()
    assert math.isnan(store.mean("lr"))
    acc = SimpleNamespace(loss_sum=torch.tensor(12.0), token_count=torch.tensor(6.0))
    s, n = aggregate_loss_metrics(acc, None, torch.device("cpu"))
    assert (float(s), float(n)) == (12.0, 6.0) and s.dtype == torch.float64


def test_token_ids_outside_the_vocabulary_are_rejected_on_the_host():
    import torch

    from nano_megatron_b200.training.trainer import check_token_ranges

    ok = {"input_ids": torch.tensor([[0, 5, 9]]), "labels": torch.tensor([[5, 9, -100]])}
    check_token_ranges(ok, 10)
    check_token_ranges(None, 10)                       # non-source ranks carry no batch
    check_token_ranges({"input_ids": torch.empty(0, dtype=torch.long)}, 10)
    with pytest.raises(ValueError, match="token id 10"):
        check_token_ranges({"input_ids": torch.tensor([[1, 10]])}, 10)
    with pytest.raises(ValueError, match="token id -1"):
        check_token_ranges({"input_ids": torch.tensor([[-1, 2]])}, 10)
    with pytest.raises(ValueError, match="labels"):
        check_token_ranges({"labels": torch.tensor([[3, 12]])}, 10)
