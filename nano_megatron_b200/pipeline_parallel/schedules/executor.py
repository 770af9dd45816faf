"""Pipeline schedule executor shared by GPipe, 1F1B and interleaved 1F1B.

Runs one rank's action plan. A forward consumes the activation received from
the previous *logical* stage (pp_rank - 1 of the same chunk, or the last rank's
previous chunk when wrapping around under interleaving), runs the stage and
sends its output to the next logical stage; a backward receives the output
gradient from the next logical stage (the last logical stage starts from its
loss), runs autograd and sends the input gradient back. Sends are always
asynchronous (up to four stay in flight, overlapping the next actions' compute):
completing each send before the next action would deadlock interleaved plans, in
which a peer may first need a transfer this rank issues later, so ``overlap_p2p``
is accepted for configuration compatibility and sends overlap either way.
Receives are posted right before the action that needs them. Semantics follow the
reference executor (src/nano_megatron/pipeline_parallel/schedules/executor.py:
270-587): loss scaled by 1/M, the last backward of each chunk marked as the
gradient-synchronising one, tied-embedding hooks around the step.
"""

from __future__ import annotations

import os

import torch

from nano_megatron_b200.utils.profiling import nvtx_range

from ..p2p import P2PCommunicator
from .base import LossAccumulator, extract_loss
from .plans import build_1f1b_plan, build_gpipe_plan, build_interleaved_plan, validate_plan

_DEBUG = os.environ.get("NMB_PP_DEBUG", "0") == "1"


class PipelineScheduleExecutor:
    def __init__(self, *, model, parallel, data_parallel, schedule: str, chunks: int,
                 activation_shape, dtype: torch.dtype, device: torch.device,
                 overlap_p2p: bool = True, dynamic_shapes: bool = False) -> None:
        self.model = model
        self.parallel = parallel
        self.dp = data_parallel
        self.schedule = schedule
        self.chunks = chunks
        self.pp = parallel.pp.size
        self.rank = parallel.coordinate.pp
        self.activation_shape = activation_shape
        self.overlap = overlap_p2p
        self.p2p = P2PCommunicator(parallel, dtype=dtype, device=device,
                                   dynamic_shapes=dynamic_shapes)
        self._warm = False

    # logical-stage helpers -------------------------------------------------
    def _logical(self, chunk: int) -> int:
        return chunk * self.pp + self.rank

    def _is_first(self, chunk: int) -> bool:
        return self._logical(chunk) == 0

    def _is_last(self, chunk: int) -> bool:
        return self._logical(chunk) == self.pp * self.chunks - 1

    def _stage(self, chunk: int):
        return self.model.chunk(chunk) if hasattr(self.model, "chunk") else self.model

    def plan(self, m: int, forward_only: bool):
        if self.schedule == "gpipe":
            plan = build_gpipe_plan(m, forward_only=forward_only)
        elif self.schedule == "1f1b":
            plan = build_1f1b_plan(m, self.pp, self.rank, forward_only=forward_only)
        else:
            plan = build_interleaved_plan(m, self.pp, self.rank, self.chunks,
                                          forward_only=forward_only)
        validate_plan(plan, m, self.chunks, forward_only)
        return plan

    def _needs_recv(self, a) -> bool:
        return (a.kind == "F" and not self._is_first(a.chunk)) or \
            (a.kind == "B" and not self._is_last(a.chunk))

    def _post(self, a):
        prev_pp = self.rank - 1  # previous logical stage lives on pp_rank-1 (mod PP)
        next_pp = self.rank + 1
        if a.kind == "F":
            return self.p2p.post_recv_activation(self.activation_shape, prev_pp,
                                                 a.microbatch, a.chunk)
        return self.p2p.post_recv_grad(self.activation_shape, next_pp, a.microbatch, a.chunk)

    def _consumer_chunk(self, chunk: int, step: int) -> int:
        """Chunk (virtual stage) of the logical stage ``step`` (+1 / -1) away."""
        return (self._logical(chunk) + step) // self.pp

    # run ------------------------------------------------------------------
    def forward_backward(self, microbatches, *, forward_only: bool = False) -> LossAccumulator:
        if not self._warm:
            self.p2p.warmup()
            self._warm = True
        m = len(microbatches)
        plan = self.plan(m, forward_only)
        acc = LossAccumulator()
        records: dict = {}
        last_b = {c: max(i for i, a in enumerate(plan) if a.kind == "B" and a.chunk == c)
                  for c in range(self.chunks)} if not forward_only else {}
        in_flight = 4
        for i, a in enumerate(plan):
            if _DEBUG:
                print(f"[pp rank {self.parallel.rank} stage {self.rank}] {a}", flush=True)
            # Receives are posted right before the action that consumes them, never
            # ahead of compute: a receive kernel left spinning on the GPU while this
            # host blocks on an implicit device synchronisation (first-use kernel
            # loading, allocator growth) can deadlock against a peer that is itself
            # blocked setting up the matching NCCL connection. Sends stay
            # asynchronous, which is what overlaps transfers with compute.
            buf = None
            if self._needs_recv(a):
                work, buf = self._post(a)
                work.wait()
            with nvtx_range(f"{a.kind} c{a.chunk} mb{a.microbatch}"):
                if a.kind == "F":
                    self._forward(a, buf, microbatches, m, acc, records, forward_only, last_b,
                                  plan)
                else:
                    self._backward(a, buf, records, is_last=(i == last_b.get(a.chunk)))
            self.p2p.drain_sends(keep=in_flight)
        self.p2p.drain_sends(keep=0)
        return acc

    def _forward(self, a, buf, microbatches, m, acc, records, forward_only, last_b, plan):
        mb = microbatches[a.microbatch]
        inp = None
        if buf is not None:
            inp = buf.requires_grad_(not forward_only)
        stage = self._stage(a.chunk)
        lb = last_b.get(a.chunk)
        sync = (not forward_only) and lb is not None and plan[lb].microbatch == a.microbatch
        if forward_only:
            with torch.no_grad():
                out = stage(inp, mb)
        else:
            with self.dp.forward_microbatch_context(synchronize_gradients=sync, unit=stage):
                out = stage(inp, mb)
        if self._is_last(a.chunk):
            out = extract_loss(out, mb, m, acc)
        else:
            self.p2p.send_activation(out, self.rank + 1, a.microbatch,
                                     self._consumer_chunk(a.chunk, +1))
        if not forward_only:
            records[(a.microbatch, a.chunk)] = (inp, out)

    def _backward(self, a, grad, records, *, is_last: bool):
        inp, out = records.pop((a.microbatch, a.chunk))
        stage = self._stage(a.chunk)
        with self.dp.microbatch_context(is_last_microbatch=is_last, unit=stage):
            if grad is None:
                torch.autograd.backward(out)
            else:
                torch.autograd.backward(out, grad)
        if inp is not None and not self._is_first(a.chunk):
            g = inp.grad if inp.grad is not None else torch.zeros_like(inp)
            self.p2p.send_grad(g, self.rank - 1, a.microbatch,
                               self._consumer_chunk(a.chunk, -1))


def build_pipeline_schedule(config, model, parallel, data_parallel):
    sched = str(getattr(config.pipeline.schedule, "value", config.pipeline.schedule))
    tp = parallel.tp.size
    sp = bool(config.parallel.sequence_parallel) and tp > 1
    seq = config.model.seq_length // parallel.cp.size
    rows = seq // tp if sp else seq
    shape = (rows, config.training.micro_batch_size, config.model.hidden_size)
    device = next(model.parameters()).device
    act = config.pipeline.activation_dtype
    if act is not None:
        dtype = {"bfloat16": torch.bfloat16, "float32": torch.float32,
                 "float16": torch.float16}[str(getattr(act, "value", act))]
    elif device.type == "cuda":
        dtype = torch.bfloat16
    else:
        dtype = next(model.parameters()).dtype
    return PipelineScheduleExecutor(
        model=model, parallel=parallel, data_parallel=data_parallel, schedule=sched,
        chunks=config.pipeline.virtual_stages_per_rank, activation_shape=shape, dtype=dtype,
        device=device, overlap_p2p=bool(config.pipeline.overlap_p2p),
        dynamic_shapes=bool(config.pipeline.dynamic_activation_shapes))
