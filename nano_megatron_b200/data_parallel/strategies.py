"""Data-parallel strategies: DDP, ZeRO-1, ZeRO-2 (ZeRO-3 lives in :mod:`.zero3`).

Trainer-facing contract of the reference's DataParallelStrategy
(src/nano_megatron/data_parallel/interface.py:17-178): ``configure_precision``,
``setup``, ``forward_microbatch_context``, ``microbatch_context``, ``backward``,
``finalize_gradients``, ``clip_grad_norm``, ``optimizer_step``,
``set_learning_rate``/``learning_rate``, ``zero_grad``, ``state_dict``/
``load_state_dict``.

B200 design:
* parameters and fp32 gradients live in flat buffers (:mod:`.buffers`); the
  weight-gradient GEMMs accumulate straight into the reduction buffer;
* the gradient reduction per bucket is one NCCL all-reduce (DDP, ZeRO-1) or
  reduce-scatter (ZeRO-2/3) of the fp32 buffer, optionally launched on a side
  stream as soon as a bucket's gradients are final (``overlap_grad_reduce``);
* averaging, clipping and AdamW are one fused kernel over the flat fp32 master
  (the clip coefficient and 1/DP are folded into its gradient scale, read on
  the device): no host synchronisation anywhere in the step;
* the updated compute-precision parameters are written by that same kernel
  (DDP) or all-gathered from the owners' shards (ZeRO).
"""

from __future__ import annotations

import contextlib

from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch import nn

from nano_megatron_b200.ops import functional as F
from nano_megatron_b200.parallel.group_plan import GroupKey

from .buffers import FlatBuffers, unique_named_parameters
from .common import clip_coefficient, local_sumsq, norm_ranges, reduce_model_parallel
from .offload import ActivationOffloader, OffloadPolicy, OptimizerStateStorage

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _torch_dtype(value) -> torch.dtype:
    name = str(getattr(value, "value", value)).lower()
    if name not in _DTYPES:
        raise ValueError(f"unsupported precision dtype: {name!r}")
    return _DTYPES[name]


class DataParallelStrategy:
    mode = "base"
    # True when forward/backward of a microbatch issues no collective and no host sync, so
    # it can be captured in a CUDA graph (gradients are reduced in finalize_gradients).
    graph_safe_microbatches = False
    # kernels.fused_dp_comm: reduce / update / gather over NVLink peer memory when the
    # replica group allows it (see replica_comm.fused_replica_supported)
    fused_replica_enabled = False
    replica = None

    def __init__(self, *, config=None, offload=None, parallel=None, parameter_domains=None) -> None:
        self.config = config
        self.parallel = parallel
        self.parameter_domains = parameter_domains
        self.offload_policy = OffloadPolicy.from_config(offload)
        self.offload_policy.validate(self.mode)
        self._activation_offloader = ActivationOffloader(self.offload_policy)
        self._model: nn.Module | None = None
        self._sync_this_backward = True
        self.param_dtype: torch.dtype | None = None
        self.compute_dtype: torch.dtype | None = None
        self.grad_reduce_dtype: torch.dtype | None = None
        self.buffers: FlatBuffers | None = None
        self._lr = 0.0
        self._lr_t: torch.Tensor | None = None
        self.step_count = 0
        self._grad_scale: torch.Tensor | None = None
        self._reduced = False
        self._pending: list = []
        self._comm_stream = None

    # ------------------------------------------------------------------ contract
    def configure_kernels(self, kernels) -> None:
        self.fused_replica_enabled = bool(getattr(kernels, "fused_dp_comm", True))

    def configure_precision(self, precision) -> None:
        self.param_dtype = _torch_dtype(precision.params)
        self.compute_dtype = _torch_dtype(precision.compute)
        self.grad_reduce_dtype = _torch_dtype(precision.grad_reduce)

    @property
    def model(self) -> nn.Module:
        if self._model is None:
            raise RuntimeError("data-parallel strategy has not been set up")
        return self._model

    @property
    def replica_group(self):
        if self.parallel is None:
            return None
        try:
            return self.parallel.group(GroupKey.DENSE_REPLICA)
        except KeyError:
            return None

    @property
    def replica_size(self) -> int:
        g = self.replica_group
        return 1 if g is None else g.size

    def _model_dtype(self, device) -> torch.dtype:
        """On CUDA the model always computes in the compute dtype (bf16) with fp32 masters."""
        compute = self.compute_dtype or torch.bfloat16
        params = self.param_dtype or compute
        if device.type == "cuda":
            return compute if compute in (torch.bfloat16, torch.float16) else torch.bfloat16
        return params if params in (torch.float32, torch.float64) else torch.float32

    def setup(self, model: nn.Module, optimizer_config, parameter_domains=None) -> nn.Module:
        self.parameter_domains = parameter_domains or self.parameter_domains
        self.optimizer_config = optimizer_config
        named = unique_named_parameters(model)
        device = named[0][1].device
        if device.type == "cpu" and torch.cuda.is_available() and False:
            device = torch.device("cuda")
        model_dtype = self._model_dtype(device)
        self._master_init = {id(p): p.detach().to(torch.float32 if p.dtype != torch.float64
                                                   else torch.float64).clone() for _, p in named}
        self._broadcast_from_replica_root(named)
        bucket_bytes = int(getattr(self.config, "bucket_bytes", 256 * 1024 * 1024))
        grad_dtype = torch.float64 if model_dtype == torch.float64 else torch.float32
        from .replica_comm import ReplicaComm, fused_replica_supported

        allocate = None
        self.replica = None
        if fused_replica_supported(self, device)[0]:
            def allocate(total, pdt, gdt):
                self.replica = ReplicaComm.create(self.replica_group, total, pdt, gdt, device)
                return self.replica.flat_tensors(total, pdt, gdt)
        self.buffers = FlatBuffers(named, domains=self.parameter_domains, parallel=self.parallel,
                                   bucket_bytes=bucket_bytes, param_dtype=model_dtype,
                                   grad_dtype=grad_dtype, device=device,
                                   unit_key=self._bucket_unit_key(), allocate=allocate)
        if self.replica is not None and any(b.group is not self.replica_group and
                                            getattr(b.group, "ranks", None) !=
                                            self.replica_group.ranks
                                            for b in self.buffers.buckets):
            raise RuntimeError("fused replica path needs every bucket on the dense replica "
                               "group")
        self._named = named
        self._ranges = norm_ranges(self.buffers, self.parallel)
        self._sp_slices = [(b, s) for b, s in self.buffers.slices() if s.sequence_parallel_grad]
        self._init_optimizer_state()
        if self.replica is not None:
            from .common import counts_toward_norm

            self.replica.prepare(self.buffers, lambda s: counts_toward_norm(s, self.parallel))
        self._lr = float(getattr(optimizer_config, "lr", 3e-4))
        self._lr_t = torch.tensor([self._lr], dtype=torch.float32, device=device)
        self._model = model
        self.overlap = bool(getattr(self.config, "overlap_grad_reduce", False))
        del self._master_init
        return model

    def _bucket_unit_key(self):
        """Optional name -> unit function forcing bucket cuts at unit boundaries."""
        return None

    def eager_last_microbatch(self) -> bool:
        """True when the last microbatch's backward communicates (overlap reducer), so a
        CUDA-graph schedule must run it eagerly."""
        return False

    def full_parameters(self):
        """Context in which every parameter holds its full value (checkpoint I/O, export).
        Only ZeRO-3 shards parameters; the other strategies always hold them whole."""
        return contextlib.nullcontext()

    def _broadcast_from_replica_root(self, named) -> None:
        g = self.replica_group
        if g is None or g.size == 1:
            return
        for _, p in named:
            dist.broadcast(p.data, src=g.ranks[0], group=g.process_group)

    @contextmanager
    def activation_context(self):
        with self._activation_offloader.context():
            yield

    @contextmanager
    def forward_microbatch_context(self, *, synchronize_gradients: bool, unit=None):
        with self.activation_context():
            yield

    @contextmanager
    def microbatch_context(self, *, is_last_microbatch: bool, unit=None):
        prev = self._sync_this_backward
        self._sync_this_backward = is_last_microbatch
        try:
            with self.activation_context():
                yield
        finally:
            self._sync_this_backward = prev

    def backward(self, loss: torch.Tensor) -> None:
        loss.backward()

    # ------------------------------------------------------------------ reduction
    def _reduce_sequence_parallel_grads(self) -> None:
        """SP norm/bias weights saw only their sequence shard: sum over TP once per step."""
        if not self._sp_slices or self.parallel is None or self.parallel.tp.size == 1:
            return
        grads = [s.parameter.main_grad for _, s in self._sp_slices]
        flat = torch.cat([g.reshape(-1) for g in grads])
        dist.all_reduce(flat, group=self.parallel.tp.process_group)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n

    def finalize_gradients(self) -> None:
        if self.replica is not None:
            return self._fused_finalize()
        # Overlapped bucket reductions finish first: the sequence-parallel norm-gradient
        # sum over TP below rewrites some of the same gradient memory (the two sums commute).
        early = self._wait_inflight()
        self._reduce_sequence_parallel_grads()
        self._reduce_buckets(skip=early)
        self._reduced = True

    def _wait_inflight(self) -> set:
        done = set()
        for idx, (work, low) in getattr(self, "_inflight", {}).items():
            work.wait()
            if low is not None:
                self.buffers.buckets[idx].grad_data.copy_(low)
            done.add(idx)
        if hasattr(self, "_inflight"):
            self._inflight.clear()
        return done

    def release_pending_work(self) -> None:
        """Wait for and drop every asynchronous reduction still referenced (shutdown)."""
        for work, _low in getattr(self, "_inflight", {}).values():
            work.wait()
        if hasattr(self, "_inflight"):
            self._inflight.clear()
        self._pending = []

    def _reduce_dtype(self) -> torch.dtype | None:
        """``precision.grad_reduce`` when it differs from the fp32 gradient buffers: the
        replica sum then runs on a copy in that dtype (as the reference packs its buckets
        in it), halving the bytes on the wire for bf16."""
        d = self.grad_reduce_dtype
        return d if d is not None and d != self.buffers.grad_dtype else None

    def _all_reduce_bucket(self, b, *, async_op: bool = False):
        """Sum bucket ``b``'s gradients over the replica group. Returns (work, low) when
        asynchronous, where ``low`` is the reduced-precision copy to copy back after the
        wait (None when the buffer itself is reduced)."""
        g = self.replica_group
        dt = self._reduce_dtype()
        target = b.grad_data if dt is None else b.grad_data.to(dt)
        work = dist.all_reduce(target, group=g.process_group, async_op=async_op)
        low = None if dt is None else target
        if async_op:
            return work, low
        if low is not None:
            b.grad_data.copy_(low)
        return None

    def _reduce_buckets(self, skip: set = frozenset()) -> None:
        g = self.replica_group
        if g is None or g.size == 1:
            return
        for b in self.buffers.buckets:
            if b.index not in skip:
                self._all_reduce_bucket(b)

    # ------------------------------------------------------------------ overlap reducer
    def _overlap_active(self) -> bool:
        g = self.replica_group
        return self.overlap and g is not None and g.size > 1

    def _register_overlap_hooks(self, model) -> None:
        """With ``overlap_grad_reduce``: buckets are cut per transformer layer, and during
        the last microbatch's backward each layer's buckets start their all-reduce (async,
        NCCL's stream) as soon as the layer's input gradient exists -- i.e. its weight
        gradients are final -- overlapping the reduction with the backward of the layers
        below. Buckets holding a tied parameter, and the embedding/head buckets, reduce in
        ``finalize_gradients`` (after the tied-embedding gradient sync), as in the
        reference's reducer (src/nano_megatron/data_parallel/buckets.py:406-525)."""
        from nano_megatron_b200.models.gpt.model import GPTLayer

        from .zero3 import unit_of_name

        names = {id(p): n for n, p in self._named}
        by_unit: dict = {}
        for b in self.buffers.buckets:
            if b.defer_until_finalize:
                continue
            by_unit.setdefault(unit_of_name(names[id(b.slices[0].parameter)]), []).append(b)
        self._inflight: dict = {}
        g = self.replica_group

        def launch(key):
            for b in by_unit.get(key, ()):
                if b.index not in self._inflight:
                    self._inflight[b.index] = self._all_reduce_bucket(b, async_op=True)

        for mod in model.modules():
            if not isinstance(mod, GPTLayer):
                continue
            key = unit_of_name(names[id(next(iter(mod.parameters())))])

            def post(_mod, args, out, key=key):
                inp = args[0] if args and isinstance(args[0], torch.Tensor) else None
                if inp is not None and inp.requires_grad and torch.is_grad_enabled():
                    def done(grad, key=key):
                        if self._sync_this_backward:
                            launch(key)
                        return grad

                    inp.register_hook(done)
                return out

            mod.register_forward_hook(post)

    def _grad_view_for_norm(self) -> tuple[torch.Tensor, list]:
        return self.buffers.grad_flat, self._ranges

    def clip_grad_norm(self, max_norm: float | None) -> torch.Tensor:
        """Global gradient norm of the *averaged* gradients (device tensor)."""
        if self.replica is not None:
            return self._fused_clip(max_norm)
        flat, ranges = self._grad_view_for_norm()
        sq = local_sumsq(flat, ranges).reshape(1).to(torch.float32)
        sq = self._reduce_norm_over_shards(sq)
        sq = reduce_model_parallel(sq, self.parallel)
        norm = sq.sqrt() / self.replica_size
        coef = clip_coefficient(norm, max_norm)
        self._grad_scale = (coef / self.replica_size).reshape(1).to(torch.float32)
        return norm.reshape(())

    def _reduce_norm_over_shards(self, sq):
        return sq

    # ------------------------------------------------------------------ fused replica path
    def _fused_finalize(self) -> None:
        """signal(GRAD), then every bucket's shard summed over the replicas in place, with
        partial squared norms (replica_comm / csrc/dp_comm.cu)."""
        from .replica_comm import CH_GRAD

        self._reduce_sequence_parallel_grads()
        self.replica.signal(CH_GRAD)
        self._replica_partials = [(b, self.replica.reduce(b, lambda x: x.offset))
                                  for b in self.buffers.buckets]
        self._reduced = True

    def materialize_reduced_gradients(self) -> None:
        """After ``finalize_gradients``: make every rank's ``main_grad`` hold the whole
        replica-summed gradient. The step itself needs only this rank's shard of each bucket
        (the fused replica path sums shards in place; ZeRO-2/3 reduce-scatter), so this
        all-gather exists for inspection and tests."""
        g = self.replica_group
        if g is None or g.size == 1 or not self._reduced or self.buffers is None:
            return
        shards = getattr(self, "shards", None)
        for i, b in enumerate(self.buffers.buckets):
            full = b.grad_data[:b.padded_numel]
            if self.replica is not None:
                mine = b.shard_view(full).clone()
            elif shards and getattr(self, "reduce_scatter", False) and full.is_cuda:
                mine = shards[i]["grad"]
            else:
                continue       # all-reduced: already whole
            dist.all_gather_into_tensor(full, mine, group=g.process_group)

    def _fused_clip(self, max_norm):
        from .common import dense_counted_here, is_dense

        dev = self.buffers.device
        dense = [p for b, p in self._replica_partials if is_dense(b)]
        expert = [p for b, p in self._replica_partials if not is_dense(b)]
        parts = [torch.cat(x).sum().reshape(1) if x else torch.zeros(1, device=dev)
                 for x in (dense, expert)]
        sq = torch.cat(parts)
        dist.all_reduce(sq, group=self.replica_group.process_group)
        if not dense_counted_here(self.parallel):
            sq[0] = 0.0          # the EP replicas of the dense parameters count once
        sq = reduce_model_parallel(sq.sum().reshape(1), self.parallel)
        norm = sq.sqrt() / self.replica_size
        coef = clip_coefficient(norm, max_norm)
        self._grad_scale = (coef / self.replica_size).reshape(1).to(torch.float32)
        return norm.reshape(())

    def _fused_optimizer_step(self) -> None:
        """AdamW over this rank's shard of every bucket with the bf16 result stored into
        every replica's parameters, then a bounded wait until all replicas have done so."""
        from .replica_comm import CH_PARAM

        if not self._reduced:
            self.finalize_gradients()
        self.step_count += 1
        b1, b2, eps, wd = self._opt_hparams()
        scale = self._scale()
        for b in self.buffers.buckets:
            master, m, v = self._shard_state(b)
            self.replica.adamw_gather(b, lambda x: x.offset, master, m, v, lr=self._lr,
                                      betas=(b1, b2), eps=eps, wd=wd, step=self.step_count,
                                      grad_scale=scale, lr_t=self._lr_t)
        self.replica.signal(CH_PARAM)
        self.replica.wait(CH_PARAM)

    def _shard_state(self, b):
        raise NotImplementedError

    # ------------------------------------------------------------------ optimizer
    def _opt_hparams(self):
        c = self.optimizer_config
        b1, b2 = tuple(getattr(c, "betas", (0.9, 0.95)))
        return (float(b1), float(b2), float(getattr(c, "eps", 1e-8)),
                float(getattr(c, "weight_decay", 0.0)))

    def set_learning_rate(self, learning_rate: float) -> None:
        self._lr = float(learning_rate)
        if self._lr_t is not None:
            self._lr_t.fill_(self._lr)

    @property
    def learning_rate(self) -> float:
        return self._lr

    def zero_grad(self) -> None:
        if self.buffers is not None:
            self.buffers.zero_grad()
        self._reduced = False
        self._grad_scale = None

    def _scale(self) -> torch.Tensor | None:
        if self._grad_scale is not None:
            return self._grad_scale
        if self.replica_size > 1:
            return torch.full((1,), 1.0 / self.replica_size, device=self.buffers.device)
        return None


class DDPStrategy(DataParallelStrategy):
    """Replicated parameters; fp32 master, exp_avg, exp_avg_sq for every element."""

    graph_safe_microbatches = True

    mode = "ddp"

    def _bucket_unit_key(self):
        if bool(getattr(self.config, "overlap_grad_reduce", False)):
            from .zero3 import unit_of_name

            return unit_of_name
        return None

    def setup(self, model, optimizer_config, parameter_domains=None):
        super().setup(model, optimizer_config, parameter_domains)
        if self._overlap_active() and self.replica is None:
            self._register_overlap_hooks(model)
        return model

    def eager_last_microbatch(self) -> bool:
        return self._overlap_active() and self.replica is None

    def _shard_state(self, b):
        lo = b.offset + b.rank * b.shard_numel
        hi = lo + b.shard_numel
        return self.master[lo:hi], self.exp_avg[lo:hi], self.exp_avg_sq[lo:hi]

    def gather_replicated_state(self) -> None:
        """Fused replica path: each rank updated only its own shards of the fp32 master and
        moments; copy every shard from its owner so the full state is current here."""
        if self.replica is None:
            return
        g = self.replica_group
        for b in self.buffers.buckets:
            for t in (self.master, self.exp_avg, self.exp_avg_sq):
                full = t[b.offset:b.offset + b.padded_numel]
                mine = full[b.rank * b.shard_numel:(b.rank + 1) * b.shard_numel].clone()
                dist.all_gather_into_tensor(full, mine, group=g.process_group)

    def _init_optimizer_state(self) -> None:
        buf = self.buffers
        self.master = torch.zeros(buf.numel, dtype=buf.grad_dtype, device=buf.device)
        for b, s in buf.slices():
            self.master[b.offset + s.start:b.offset + s.end].copy_(
                self._master_init[id(s.parameter)].reshape(-1))
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)

    def optimizer_step(self) -> None:
        if self.replica is not None:
            return self._fused_optimizer_step()
        if not self._reduced:
            self.finalize_gradients()
        self.step_count += 1
        b1, b2, eps, wd = self._opt_hparams()
        low = self.buffers.param_flat if self.buffers.param_flat.dtype != self.master.dtype else None
        F.adamw_(self.master, self.buffers.grad_flat, self.exp_avg, self.exp_avg_sq, low,
                 lr=self._lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd,
                 step=self.step_count, grad_scale=self._scale(), lr_t=self._lr_t)
        if low is None:
            self.buffers.param_flat.copy_(self.master)

    def state_dict(self) -> dict:
        """torch.optim.AdamW-shaped state (one entry per unique parameter) + fp32 masters."""
        self.gather_replicated_state()
        b1, b2, eps, wd = self._opt_hparams()
        state, ids = {}, []
        for i, (b, s) in enumerate(self.buffers.slices()):
            a, e = b.offset + s.start, b.offset + s.end
            shape = s.parameter.shape
            state[i] = {"step": torch.tensor(float(self.step_count)),
                        "exp_avg": self.exp_avg[a:e].view(shape).detach().cpu().clone(),
                        "exp_avg_sq": self.exp_avg_sq[a:e].view(shape).detach().cpu().clone(),
                        "master_param": self.master[a:e].view(shape).detach().cpu().clone()}
            ids.append(i)
        groups = [{"lr": self._lr, "betas": (b1, b2), "eps": eps, "weight_decay": wd,
                   "amsgrad": False, "maximize": False, "foreach": None, "capturable": False,
                   "differentiable": False, "fused": None, "params": ids}]
        return {"mode": self.mode, "optimizer": {"state": state, "param_groups": groups}}

    def load_state_dict(self, state_dict) -> None:
        if state_dict.get("mode") != self.mode:
            raise ValueError(f"data-parallel state mode {state_dict.get('mode')!r} does not "
                             f"match {self.mode!r}")
        opt = state_dict["optimizer"]
        for i, (b, s) in enumerate(self.buffers.slices()):
            a, e = b.offset + s.start, b.offset + s.end
            st = opt["state"].get(i) or opt["state"].get(str(i))
            if st is None:
                continue
            self.exp_avg[a:e].copy_(st["exp_avg"].reshape(-1))
            self.exp_avg_sq[a:e].copy_(st["exp_avg_sq"].reshape(-1))
            if "master_param" in st:
                self.master[a:e].copy_(st["master_param"].reshape(-1))
            else:
                self.master[a:e].copy_(s.parameter.detach().reshape(-1).float())
            self.step_count = int(float(st["step"]))
        self._lr = float(opt["param_groups"][0]["lr"])
        self.set_learning_rate(self._lr)
        self.sync_params_from_master()

    def sync_params_from_master(self) -> None:
        self.buffers.param_flat.copy_(self.master)

    def load_model_parameters(self) -> None:
        """Refresh the fp32 masters after parameters were overwritten (checkpoint load)."""
        for b, s in self.buffers.slices():
            self.master[b.offset + s.start:b.offset + s.end].copy_(
                s.parameter.detach().reshape(-1))


class ReplicatedStrategy(DDPStrategy):
    """DDP semantics without a replica group (single replica)."""

    mode = "replicated"


class FlatShardZeROStrategy(DataParallelStrategy):
    """ZeRO-1/2: fp32 master + Adam moments sharded over the replica group."""

    graph_safe_microbatches = True
    mode = "zero"
    reduce_scatter = False

    def _init_optimizer_state(self) -> None:
        buf = self.buffers
        storage = OptimizerStateStorage(self.offload_policy, buf.device)
        self.shards = []
        for b in buf.buckets:
            full = torch.zeros(b.padded_numel, dtype=buf.grad_dtype)
            for s in b.slices:
                full[s.start:s.end].copy_(self._master_init[id(s.parameter)].reshape(-1).cpu())
            lo, hi = b.rank * b.shard_numel, (b.rank + 1) * b.shard_numel
            master = storage.zeros(b.shard_numel).to(buf.grad_dtype)
            master.copy_(full[lo:hi])
            if not self.offload_policy.optimizer_state:
                master = master.to(buf.device)
            self.shards.append({"master": master, "exp_avg": storage.zeros(b.shard_numel),
                                "exp_avg_sq": storage.zeros(b.shard_numel),
                                "grad": torch.zeros(b.shard_numel, dtype=buf.grad_dtype,
                                                    device=buf.device)})

    def _reduce_buckets(self, skip: set = frozenset()) -> None:
        g = self.replica_group
        for b, sh in zip(self.buffers.buckets, self.shards):
            full = b.grad_data[:b.padded_numel]
            if g is None or g.size == 1:
                sh["grad"].copy_(full)
                continue
            dt = self._reduce_dtype()
            if dt is not None:
                full = full.to(dt)
            if self.reduce_scatter and full.is_cuda:
                out = sh["grad"] if dt is None else torch.empty(sh["grad"].shape, dtype=dt,
                                                                 device=full.device)
                dist.reduce_scatter_tensor(out, full, group=g.process_group)
                if dt is not None:
                    sh["grad"].copy_(out)
            else:
                dist.all_reduce(full, group=g.process_group)
                sh["grad"].copy_(b.shard_view(full))

    def _grad_view_for_norm(self):
        # squared norm over this rank's shard of each bucket (counting rule per slice)
        return None, None

    def _shard_state(self, b):
        sh = self.shards[b.index]
        return sh["master"], sh["exp_avg"], sh["exp_avg_sq"]

    def clip_grad_norm(self, max_norm: float | None) -> torch.Tensor:
        if self.replica is not None:
            return self._fused_clip(max_norm)
        dev = self.buffers.device
        sq = torch.zeros(2, dtype=torch.float32, device=dev)   # [dense, expert] shard sums
        from .common import counts_toward_norm, dense_counted_here, is_dense

        for b, sh in zip(self.buffers.buckets, self.shards):
            lo = b.rank * b.shard_numel
            hi = lo + b.shard_numel
            slot = 0 if is_dense(b) else 1
            for s in b.slices:
                a, e = max(s.start, lo), min(s.end, hi)
                if a >= e or not counts_toward_norm(s, self.parallel):
                    continue
                sq[slot] += F.sumsq(sh["grad"][a - lo:e - lo])
        g = self.replica_group
        if g is not None and g.size > 1:
            dist.all_reduce(sq, group=g.process_group)
        if not dense_counted_here(self.parallel):
            sq[0] = 0.0          # the EP replicas of the dense parameters count once
        sq = reduce_model_parallel(sq.sum().reshape(1), self.parallel)
        norm = sq.sqrt() / self.replica_size
        coef = clip_coefficient(norm, max_norm)
        self._grad_scale = (coef / self.replica_size).reshape(1).to(torch.float32)
        return norm.reshape(())

    def optimizer_step(self) -> None:
        if self.replica is not None:
            return self._fused_optimizer_step()
        if not self._reduced:
            self.finalize_gradients()
        self.step_count += 1
        b1, b2, eps, wd = self._opt_hparams()
        g = self.replica_group
        scale = self._scale()
        for b, sh in zip(self.buffers.buckets, self.shards):
            dev = sh["master"].device
            grad = sh["grad"] if dev == sh["grad"].device else sh["grad"].to(dev)
            sc = scale if scale is None or scale.device == dev else scale.to(dev)
            lr_t = self._lr_t if self._lr_t.device == dev else None
            F.adamw_(sh["master"], grad, sh["exp_avg"], sh["exp_avg_sq"], None, lr=self._lr,
                     beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=self.step_count,
                     grad_scale=sc, lr_t=lr_t)
            low = sh["master"].to(device=b.param_data.device, dtype=b.param_data.dtype)
            full = b.param_data[:b.padded_numel]
            if g is None or g.size == 1:
                full.copy_(low)
            elif full.is_cuda:
                dist.all_gather_into_tensor(full, low, group=g.process_group)
            else:
                parts = [torch.empty_like(low) for _ in range(g.size)]
                dist.all_gather(parts, low, group=g.process_group)
                full.copy_(torch.cat(parts))

    def _gather_shard(self, b, t: torch.Tensor) -> torch.Tensor:
        g = self.replica_group
        if g is None or g.size == 1:
            return t.detach().cpu().clone()
        parts = [torch.empty_like(t) for _ in range(g.size)]
        dist.all_gather(parts, t.contiguous(), group=g.process_group)
        return torch.cat(parts).cpu()

    def state_dict(self) -> dict:
        buckets = {}
        for b, sh in zip(self.buffers.buckets, self.shards):
            entry = {"metadata": b.metadata()}
            for k, key in (("master", "master_parameter"), ("exp_avg", "exp_avg"),
                           ("exp_avg_sq", "exp_avg_sq")):
                t = sh[k].to(self.buffers.device) if sh[k].device != self.buffers.device \
                    else sh[k]
                entry[key] = self._gather_shard(b, t)[:b.numel].clone()
            buckets[str(b.index)] = entry      # string keys, as the reference's loader reads
        return {"mode": self.mode, "step": self.step_count, "learning_rate": self._lr,
                "buckets": buckets}

    def load_state_dict(self, state_dict) -> None:
        if state_dict.get("mode") != self.mode:
            raise ValueError(f"data-parallel state mode {state_dict.get('mode')!r} does not "
                             f"match {self.mode!r}")
        self.step_count = int(state_dict["step"])
        self.set_learning_rate(float(state_dict["learning_rate"]))
        for b, sh in zip(self.buffers.buckets, self.shards):
            entry = state_dict["buckets"].get(b.index) or state_dict["buckets"].get(str(b.index))
            meta = entry["metadata"]
            if meta["parameter_names"] != [s.name for s in b.slices] or meta["numel"] != b.numel:
                raise ValueError("zero bucket boundaries must match the checkpoint")
            lo = b.rank * b.shard_numel
            for k, key in (("master", "master_parameter"), ("exp_avg", "exp_avg"),
                           ("exp_avg_sq", "exp_avg_sq")):
                full = torch.zeros(b.padded_numel, dtype=sh[k].dtype)
                full[:b.numel].copy_(entry[key].reshape(-1)[:b.numel])
                sh[k].copy_(full[lo:lo + b.shard_numel])
        self.sync_params_from_master()

    def sync_params_from_master(self) -> None:
        g = self.replica_group
        for b, sh in zip(self.buffers.buckets, self.shards):
            low = sh["master"].to(device=b.param_data.device, dtype=b.param_data.dtype)
            full = b.param_data[:b.padded_numel]
            if g is None or g.size == 1:
                full.copy_(low)
            else:
                parts = [torch.empty_like(low) for _ in range(g.size)]
                dist.all_gather(parts, low, group=g.process_group)
                full.copy_(torch.cat(parts))

    def load_model_parameters(self) -> None:
        for b, sh in zip(self.buffers.buckets, self.shards):
            lo = b.rank * b.shard_numel
            src = b.param_data[:b.padded_numel][lo:lo + b.shard_numel]
            sh["master"].copy_(src.to(sh["master"].dtype))


class Zero1Strategy(FlatShardZeROStrategy):
    mode = "zero1"
    reduce_scatter = False


class Zero2Strategy(FlatShardZeROStrategy):
    mode = "zero2"
    reduce_scatter = True
