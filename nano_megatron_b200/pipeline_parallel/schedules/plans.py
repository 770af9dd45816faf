"""Per-rank action plans of the pipeline schedules.

An action is ``(kind, microbatch, chunk)`` with kind ``"F"`` or ``"B"``. Same
orders as the reference (src/nano_megatron/pipeline_parallel/schedules/
gpipe.py:19-34, one_f_one_b.py:19-72, interleaved.py:20-98):

* GPipe: every forward in order, then every backward in reverse order;
* 1F1B: ``min(PP - rank - 1, M)`` warm-up forwards, then alternate F/B, then
  drain the remaining backwards;
* interleaved 1F1B (``v`` chunks per rank, M % PP == 0): virtual step k maps to
  chunk ``(k // PP) % v`` (reversed for backward) and microbatch
  ``(k // (PP*v)) * PP + k % PP``; warm-up ``(PP - rank - 1) * 2 + (v - 1) * PP``.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Action:
    kind: str        # "F" or "B"
    microbatch: int
    chunk: int = 0


def build_gpipe_plan(num_microbatches: int, *, forward_only: bool = False) -> list[Action]:
    plan = [Action("F", m) for m in range(num_microbatches)]
    if not forward_only:
        plan += [Action("B", m) for m in reversed(range(num_microbatches))]
    return plan


def build_1f1b_plan(num_microbatches: int, pipeline_size: int, pipeline_rank: int, *,
                    forward_only: bool = False) -> list[Action]:
    m = num_microbatches
    if forward_only:
        return [Action("F", i) for i in range(m)]
    warm = min(pipeline_size - pipeline_rank - 1, m)
    plan = [Action("F", i) for i in range(warm)]
    for i in range(m - warm):
        plan.append(Action("F", warm + i))
        plan.append(Action("B", i))
    plan += [Action("B", i) for i in range(m - warm, m)]
    return plan


def _virtual(k: int, pp: int, v: int, *, forward: bool) -> tuple[int, int]:
    group = pp * v
    chunk = (k // pp) % v
    if not forward:
        chunk = v - 1 - chunk
    mb = (k // group) * pp + k % pp
    return mb, chunk


def build_interleaved_schedule_table(num_microbatches: int, pipeline_size: int,
                                     virtual_stages: int) -> list[tuple[int, int]]:
    """Forward virtual-step order as (microbatch, chunk)."""
    if num_microbatches % pipeline_size:
        raise ValueError("interleaved 1F1B requires microbatches divisible by pipeline size")
    return [_virtual(k, pipeline_size, virtual_stages, forward=True)
            for k in range(num_microbatches * virtual_stages)]


def build_interleaved_plan(num_microbatches: int, pipeline_size: int, pipeline_rank: int,
                           virtual_stages: int, *, forward_only: bool = False) -> list[Action]:
    m, pp, v = num_microbatches, pipeline_size, virtual_stages
    total = m * v
    if forward_only:
        # forwards in groups of min(PP, M) microbatches per chunk
        plan = []
        g = min(pp, m)
        for start in range(0, m, g):
            for c in range(v):
                for mb in range(start, min(start + g, m)):
                    plan.append(Action("F", mb, c))
        return plan
    if m % pp:
        raise ValueError("interleaved 1F1B requires gradient_accumulation_steps % PP == 0")
    warm = min((pp - pipeline_rank - 1) * 2 + (v - 1) * pp, total)
    plan = []
    for k in range(warm):
        mb, c = _virtual(k, pp, v, forward=True)
        plan.append(Action("F", mb, c))
    for i in range(total - warm):
        mb, c = _virtual(warm + i, pp, v, forward=True)
        plan.append(Action("F", mb, c))
        mb, c = _virtual(i, pp, v, forward=False)
        plan.append(Action("B", mb, c))
    for i in range(total - warm, total):
        mb, c = _virtual(i, pp, v, forward=False)
        plan.append(Action("B", mb, c))
    return plan


def validate_plan(plan: list[Action], num_microbatches: int, chunks: int = 1,
                  forward_only: bool = False) -> None:
    seen_f, seen_b = set(), set()
    for a in plan:
        key = (a.microbatch, a.chunk)
        if a.kind == "F":
            if key in seen_f:
                raise ValueError(f"duplicate forward {key}")
            seen_f.add(key)
        else:
            if key not in seen_f or key in seen_b:
                raise ValueError(f"backward {key} before its forward or duplicated")
            seen_b.add(key)
    want = {(m, c) for m in range(num_microbatches) for c in range(chunks)}
    if seen_f != want or (not forward_only and seen_b != want):
        raise ValueError("plan does not cover every (microbatch, chunk) exactly once")
