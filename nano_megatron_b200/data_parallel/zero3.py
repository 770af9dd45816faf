"""ZeRO-3: parameters, gradients and optimizer state sharded over the replica group.

Sharding units are the transformer layers (one unit per ``GPTLayer``) plus one
"outer" unit holding everything else (embedding, final norm, LM head);
buckets are cut at unit boundaries so a unit is a whole number of buckets.
Between uses a rank keeps only its bf16 shard of every bucket (and the fp32
master / Adam moment shards of ZeRO-1/2); the full bf16 parameters exist only
while their unit computes:

* a layer's pre-forward hook all-gathers its buckets into fresh buffers and
  points the parameters' ``.data`` at them (the next layer's gather is started
  asynchronously at the same time, so it overlaps this layer's compute); the
  post-forward hook releases them again when ``reshard_after_forward``;
* in the backward pass a hook on the layer's output gathers the unit again
  (prefetching the layer before it) and a hook on its input releases it once
  the input gradient exists;
* the outer unit is gathered at the stage's first forward and released when
  the gradients are finalised.

Gradients accumulate in the full fp32 ``main_grad`` buffer over the
microbatches and are reduce-scattered to the owners once per step; each owner
runs the sharded AdamW and refreshes its bf16 shard from the fp32 master. The
reference wraps the whole stage (or each virtual chunk) in one FSDP2 unit
instead (src/nano_megatron/data_parallel/zero3.py:152-165), which gathers
every parameter of the stage at once.

``offload.zero3_params_and_grads`` (the reference's FSDP2 ``CPUOffloadPolicy``,
src/nano_megatron/data_parallel/zero3.py:77-80,139-142) keeps every sharded tensor in
(pinned) host memory: the bf16 parameter shards, the reduced fp32 gradient shards, the
fp32 masters and both Adam moments. A gather copies the shard to the device first (an
asynchronous copy from pinned memory on the compute stream, which the all-gather then
follows); after the reduce-scatter each gradient shard is copied to the host, and the
AdamW update runs on the host. What stays on the device between uses is the flat fp32
gradient accumulation buffer of the microbatches, as without offload.
"""

from __future__ import annotations

import re
from contextlib import contextmanager

import torch
import torch.distributed as dist

from .strategies import Zero2Strategy

_LAYER = re.compile(r"(?:^|\.)layers\.(\d+)\.")
_CHUNK = re.compile(r"^chunks\.(\d+)\.")


def unit_of_name(name: str):
    """Sharding unit of a parameter: ("layer", chunk, local index) or "outer"."""
    m = _LAYER.search(name)
    if m is None:
        return "outer"
    c = _CHUNK.match(name)
    return ("layer", int(c.group(1)) if c else 0, int(m.group(1)))


class Zero3Strategy(Zero2Strategy):
    mode = "zero3"
    graph_safe_microbatches = False
    reduce_scatter = True

    # ------------------------------------------------------------------ setup
    def _bucket_unit_key(self):
        return unit_of_name

    def setup(self, model, optimizer_config, parameter_domains=None):
        super().setup(model, optimizer_config, parameter_domains)
        buf = self.buffers
        names = {id(p): n for n, p in self._named}
        self._units: dict = {}
        for b in buf.buckets:
            key = unit_of_name(names[id(b.slices[0].parameter)])
            self._units.setdefault(key, []).append(b)
            b.shapes = [tuple(s.parameter.shape) for s in b.slices]
            b.bf16_shard = b.shard_view(b.param_data[:b.padded_numel]).clone()
        self.host_shards = bool(self.offload_policy.zero3_params_and_grads)
        if self.host_shards:
            self._move_shards_to_host()
        self._empty = torch.empty(0, dtype=buf.param_dtype, device=buf.device)
        self._gathered: set = set()
        self._pending: dict = {}
        self._in_backward: set = set()
        # Drop the full parameter storage: from here on it exists only per gathered unit.
        for b in buf.buckets:
            b.param_data = None
            for s in b.slices:
                s.parameter.data = self._empty
        buf.param_flat = None
        self._register_hooks(model)
        return model

    def _move_shards_to_host(self) -> None:
        pin = bool(self.offload_policy.pin_memory) and torch.cuda.is_available()

        def host(t: torch.Tensor) -> torch.Tensor:
            out = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin)
            out.copy_(t)
            return out

        for b, sh in zip(self.buffers.buckets, self.shards):
            b.bf16_shard = host(b.bf16_shard)
            for k in ("master", "exp_avg", "exp_avg_sq"):
                sh[k] = host(sh[k])
            sh["host_grad"] = host(sh["grad"])

    def _layer_modules(self, model):
        from nano_megatron_b200.models.gpt.model import GPTLayer

        names = {id(p): n for n, p in self._named}
        out = []
        for mod in model.modules():
            if isinstance(mod, GPTLayer):
                first = next(iter(mod.parameters()))
                out.append((unit_of_name(names[id(first)]), mod))
        return out

    def _register_hooks(self, model) -> None:
        layers = self._layer_modules(model)
        order = [k for k, _ in layers]
        nxt = {order[i]: order[i + 1] for i in range(len(order) - 1)}
        prv = {order[i]: order[i - 1] for i in range(1, len(order))}

        from nano_megatron_b200.models.gpt.model import GPTModel

        def stage_pre(_mod, _args, _kwargs):
            self.gather("outer")

        for mod in model.modules():
            if isinstance(mod, GPTModel):
                mod.register_forward_pre_hook(stage_pre, with_kwargs=True)
        for key, mod in layers:
            def pre(_mod, _args, key=key):
                self.gather(key)
                if key in nxt:
                    self.prefetch(nxt[key])

            def post(_mod, args, out, key=key):
                reshard = bool(getattr(self.config, "reshard_after_forward", True))
                if isinstance(out, torch.Tensor) and out.requires_grad:
                    def before_backward(grad, key=key):
                        self.gather(key)
                        self._in_backward.add(key)
                        if key in prv:
                            self.prefetch(prv[key])
                        return grad

                    out.register_hook(before_backward)
                    inp = args[0] if args and isinstance(args[0], torch.Tensor) else None
                    if inp is not None and inp.requires_grad:
                        inp.register_hook(lambda g, key=key: (self._end_backward(key), g)[1])
                # A forward re-run by activation checkpointing inside this unit's backward
                # must keep the parameters its backward is about to use.
                if (reshard or not torch.is_grad_enabled()) and key not in self._in_backward:
                    self.release(key)
                return out

            mod.register_forward_pre_hook(pre)
            mod.register_forward_hook(post)

    # ------------------------------------------------------------------ gather / release
    def _start_gather(self, b, async_op: bool):
        full = torch.empty(b.storage_numel, dtype=self.buffers.param_dtype,
                           device=self.buffers.device)
        shard = b.bf16_shard
        if shard.device != full.device:          # host-resident shard: stage it first
            shard = shard.to(full.device, non_blocking=True)
        g = self.replica_group
        if g is None or g.size == 1:
            full[:b.padded_numel].copy_(shard)
            return full, None
        work = dist.all_gather_into_tensor(full[:b.padded_numel], shard,
                                           group=g.process_group, async_op=async_op)
        return full, work

    def prefetch(self, key) -> None:
        if key in self._gathered or key in self._pending or key not in self._units:
            return
        self._pending[key] = [self._start_gather(b, True) for b in self._units[key]]

    def gather(self, key) -> None:
        if key in self._gathered or key not in self._units:
            return
        started = self._pending.pop(key, None)
        if started is None:
            started = [self._start_gather(b, False) for b in self._units[key]]
        for b, (full, work) in zip(self._units[key], started):
            if work is not None:
                work.wait()
            b.param_data = full
            for s, shape in zip(b.slices, b.shapes):
                s.parameter.data = full[s.start:s.end].view(shape)
        self._gathered.add(key)

    def _end_backward(self, key) -> None:
        self._in_backward.discard(key)
        self.release(key)

    def release(self, key) -> None:
        if key not in self._gathered:
            return
        for b in self._units[key]:
            b.param_data = None
            for s in b.slices:
                s.parameter.data = self._empty
        self._gathered.discard(key)

    def release_all(self) -> None:
        self._in_backward.clear()
        for key in list(self._gathered):
            self.release(key)
        for key, started in list(self._pending.items()):
            for _, work in started:
                if work is not None:
                    work.wait()
        self._pending.clear()

    @contextmanager
    def full_parameters(self):
        """Gather every unit; on exit, keep any parameter values written meanwhile (e.g. a
        checkpoint's model state) by copying this rank's part back into its shard."""
        for key in self._units:
            self.gather(key)
        try:
            yield
        finally:
            for b in self.buffers.buckets:
                b.bf16_shard.copy_(b.shard_view(b.param_data[:b.padded_numel]))
            self.release_all()

    # ------------------------------------------------------------------ step
    def finalize_gradients(self) -> None:
        super().finalize_gradients()
        self.release_all()

    def optimizer_step(self) -> None:
        if not self._reduced:
            self.finalize_gradients()
        self.step_count += 1
        b1, b2, eps, wd = self._opt_hparams()
        scale = self._scale()
        from nano_megatron_b200.ops import functional as F

        for b, sh in zip(self.buffers.buckets, self.shards):
            dev = sh["master"].device
            if "host_grad" in sh:
                sh["host_grad"].copy_(sh["grad"])          # the reduced shard, to the host
                grad = sh["host_grad"]
            else:
                grad = sh["grad"] if dev == sh["grad"].device else sh["grad"].to(dev)
            sc = scale if scale is None or scale.device == dev else scale.to(dev)
            lr_t = self._lr_t if self._lr_t.device == dev else None
            F.adamw_(sh["master"], grad, sh["exp_avg"], sh["exp_avg_sq"], None, lr=self._lr,
                     beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=self.step_count,
                     grad_scale=sc, lr_t=lr_t)
            b.bf16_shard.copy_(sh["master"].to(device=b.bf16_shard.device,
                                               dtype=b.bf16_shard.dtype))

    def sync_params_from_master(self) -> None:
        self.release_all()
        for b, sh in zip(self.buffers.buckets, self.shards):
            b.bf16_shard.copy_(sh["master"].to(device=b.bf16_shard.device,
                                               dtype=b.bf16_shard.dtype))

    def load_model_parameters(self) -> None:
        with self.full_parameters():
            for b, sh in zip(self.buffers.buckets, self.shards):
                sh["master"].copy_(b.shard_view(b.param_data[:b.padded_numel])
                                   .to(sh["master"].dtype))
