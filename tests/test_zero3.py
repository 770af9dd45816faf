"""ZeRO-3 parameter sharding (gloo, CPU): parameters exist only while their unit runs,
and training matches DDP step for step, with and without the host-resident shards of
``offload.zero3_params_and_grads``. Reference counterpart:
tests/distributed_cpu/test_zero3_fsdp2.py."""

from __future__ import annotations

import os

import pytest
import torch

from dist_utils import run_ranks

pytestmark = pytest.mark.distributed


def _cfg(mode: str, ac: str = "none", offload: bool = False):
    from nano_megatron_b200.config import config_from_dict

    return config_from_dict({
        "model": {"layers": 3, "hidden_size": 32, "ffn_hidden_size": 64, "heads": 4,
                  "kv_heads": 2, "seq_length": 16, "vocab_size": 96},
        "parallel": {"tensor": 1, "pipeline": 1, "context": 1, "expert": 1, "data": 2},
        "precision": {"params": "float32", "compute": "float32"},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 2, "seed": 3},
        "data_parallel": {"mode": mode, "bucket_bytes": 4096},
        "activation_checkpoint": {"mode": ac},
        "offload": {"zero3_params_and_grads": offload},
        "optimizer": {"lr": 1e-2, "clip_grad_norm": 1.0}})


def _worker(rank, world, out_dir, ac):
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    res = {}
    for mode in ("ddp", "zero3", "zero3_offload"):
        cfg = _cfg(mode.split("_")[0], ac, offload=mode.endswith("offload"))
        rt = DistributedRuntime(cfg.distributed).initialize()
        torch.manual_seed(0)
        comps = build_training_components(cfg, rt)
        tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                     data_parallel=comps.data_parallel, rng=comps.rng)
        dp = comps.data_parallel
        if mode.startswith("zero3"):
            assert all(p.numel() == 0 for p in comps.model.parameters())
            assert dp.host_shards == (mode == "zero3_offload")
            if dp.host_shards:    # every sharded tensor lives in host memory
                for b, sh in zip(dp.buffers.buckets, dp.shards):
                    assert b.bf16_shard.device.type == "cpu"
                    assert {sh[k].device.type for k in ("master", "exp_avg", "exp_avg_sq",
                                                        "host_grad")} == {"cpu"}
            units = dp._units
            assert sum(isinstance(k, tuple) for k in units) == 3   # one unit per layer
        losses = []
        for step in range(3):
            g = torch.Generator().manual_seed(50 + step)
            ids = torch.randint(0, 96, (8, 17), generator=g)[rank * 4:(rank + 1) * 4]
            out = tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
            losses.append(float(out["loss_sum"] / out["token_count"]))
            if mode.startswith("zero3"):
                assert all(p.numel() == 0 for p in comps.model.parameters())
        with dp.full_parameters():
            params = {n: p.detach().clone() for n, p in comps.model.named_parameters()}
        res[mode] = (losses, params)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))


@pytest.mark.parametrize("ac", ["none", "full"])
def test_zero3_matches_ddp(tmp_path, ac):
    run_ranks(2, _worker, str(tmp_path), ac)
    for r in range(2):
        res = torch.load(tmp_path / f"r{r}.pt")
        l0, p0 = res["ddp"]
        for mode in ("zero3", "zero3_offload"):
            l1, p1 = res[mode]
            for a, b in zip(l0, l1):
                assert abs(a - b) < 1e-5 * abs(a), (mode, l0, l1)
            for n in p0:
                torch.testing.assert_close(p1[n], p0[n], rtol=1e-5, atol=1e-6)
