"""Parallel layouts on several GPUs (NCCL, bf16, sm_100a kernels) reproduce one GPU.

The GPU counterpart of the gloo equivalence tests: a TP1/PP1/DP1 model on one GPU defines
the weights and the reference loss and gradients of one training step; every layout
loads its shard of the same weights on 2 (or 4) GPUs, runs the step on the same global
batch, and its token-weighted loss and merged gradients must agree within bf16
tolerance. Covers the NCCL paths the single-GPU tests cannot: pipeline P2P (1F1B and
interleaved), context-parallel ring (zig-zag) and all-gather, the overlapped DDP
reducer, ZeRO-1, ZeRO-2 and ZeRO-3 (also with its shards offloaded to pinned host
memory). Child processes, one per GPU, NVLS off, bounded by timeouts.
"""

from __future__ import annotations

import os

import pytest
import torch

from dist_utils import run_gpu_ranks
from test_parallel_equivalence_gloo import _global_name

pytestmark = pytest.mark.gpu

MODEL = {"layers": 4, "hidden_size": 256, "ffn_hidden_size": 512, "heads": 4, "kv_heads": 2,
         "seq_length": 256, "vocab_size": 1024}
MB, GB = 2, 8


def _config(layout: dict):
    from nano_megatron_b200.config import config_from_dict

    par = {"tensor": 1, "pipeline": 1, "context": 1, "expert": 1, "data": 1,
           "sequence_parallel": False}
    par.update(layout.get("parallel", {}))
    dp = par["data"]
    return config_from_dict({
        "model": dict(MODEL), "parallel": par,
        "precision": {"params": "bfloat16", "compute": "bfloat16", "grad_reduce": "float32"},
        "distributed": {"device": "cuda", "backend": "nccl", "timeout_minutes": 2},
        "kernels": {"backend": "b200", "cuda_graphs": False},
        "training": {"micro_batch_size": MB, "gradient_accumulation_steps": GB // (MB * dp)},
        "data_parallel": {"mode": layout.get("dp_mode", "ddp"),
                          "overlap_grad_reduce": layout.get("dp_overlap", False),
                          "bucket_bytes": 1 << 18 if layout.get("dp_overlap") else 1 << 28},
        "pipeline": layout.get("pipeline", {}),
        "context_parallel": layout.get("cp", {}),
        "offload": {"zero3_params_and_grads": bool(layout.get("offload"))},
        "optimizer": {"lr": 1e-3, "clip_grad_norm": None}})


def _batch():
    g = torch.Generator().manual_seed(99)
    ids = torch.randint(0, MODEL["vocab_size"], (GB, MODEL["seq_length"] + 1), generator=g)
    return {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}


def _step(cfg, out_path, full_path=None):
    """One forward/backward of the global batch; saves loss and merged-ready gradients."""
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components
    from nano_megatron_b200.training.metrics import aggregate_loss_metrics
    from nano_megatron_b200.utils.sharding import shard_tensor, tensor_shard_dim

    rt = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, rt)
    parts = getattr(comps.built, "partitions", None) or (comps.built.partition,)
    tp = comps.parallel.tp
    if full_path is None:
        # state_dict (not named_parameters): a tied LM head keeps its own key for PP stages
        full = {k[len("model."):]: v.detach().float().cpu().clone()
                for k, v in comps.model.state_dict().items()}
        torch.save(full, out_path + ".weights")
    else:
        full = torch.load(full_path)
        with torch.no_grad():
            for name, p in comps.model.named_parameters():
                g = _global_name(name, parts)
                p.copy_(shard_tensor(full[g], tensor_shard_dim(g), tp.rank, tp.size))
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng, device=rt.device)
    batch = _batch()
    c = comps.parallel.coordinate
    dp_size = comps.parallel.dp.size
    rows = GB // dp_size
    local = {k: v[c.dp * rows:(c.dp + 1) * rows] for k, v in batch.items()}
    micro = tr._prepare_batch(local if tr.batch_router.is_source else None)
    dp = comps.data_parallel
    dp.zero_grad()
    acc = tr.schedule.forward_backward(micro)
    comps.model.synchronize_tied_embedding_gradients()
    dp.finalize_gradients()
    dp.materialize_reduced_gradients()
    s, n = aggregate_loss_metrics(acc, comps.parallel, rt.device)
    grads, seen = {}, set()
    for name, p in comps.model.named_parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        grads[_global_name(name, parts)] = (p.main_grad.float() / dp.replica_size).cpu()
    from nano_megatron_b200.ops._ext import check_status

    check_status(rt.device)
    torch.save({"loss": float(s / n), "grads": grads, "tp_rank": tp.rank, "tp": tp.size,
                "dp_rank": c.dp}, out_path)
    comps.close(tr)


def _single_rank(rank, world, out_dir):
    _step(_config({}), os.path.join(out_dir, "single.pt"))


def _layout_rank(rank, world, layout, out_dir):
    _step(_config(layout), os.path.join(out_dir, f"rank{rank}.pt"),
          full_path=os.path.join(out_dir, "single.pt.weights"))


LAYOUTS = {
    "pp2_1f1b": ({"parallel": {"pipeline": 2},
                  "pipeline": {"schedule": "1f1b", "overlap_p2p": True}}, 2),
    "pp2_interleaved": ({"parallel": {"pipeline": 2},
                         "pipeline": {"schedule": "interleaved_1f1b",
                                      "virtual_stages_per_rank": 2}}, 2),
    "cp2_ring_zigzag": ({"parallel": {"context": 2},
                         "cp": {"backend": "ring", "load_balance": True}}, 2),
    "cp2_all_gather": ({"parallel": {"context": 2}, "cp": {"backend": "all_gather"}}, 2),
    "dp2_ddp_overlap": ({"parallel": {"data": 2}, "dp_overlap": True}, 2),
    "dp2_zero1": ({"parallel": {"data": 2}, "dp_mode": "zero1"}, 2),
    "dp2_zero2": ({"parallel": {"data": 2}, "dp_mode": "zero2"}, 2),
    "dp2_zero3": ({"parallel": {"data": 2}, "dp_mode": "zero3"}, 2),
    "dp2_zero3_offload": ({"parallel": {"data": 2}, "dp_mode": "zero3", "offload": True}, 2),
    "tp2_sp": ({"parallel": {"tensor": 2, "sequence_parallel": True}}, 2),
    "tp2_pp2_sp": ({"parallel": {"tensor": 2, "pipeline": 2, "sequence_parallel": True}}, 4),
    "tp2_cp2_sp_ring": ({"parallel": {"tensor": 2, "context": 2, "sequence_parallel": True},
                         "cp": {"backend": "ring", "load_balance": True}}, 4),
}


@pytest.fixture(scope="module")
def single(tmp_path_factory):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs at least 2 GPUs")
    d = str(tmp_path_factory.mktemp("single_gpu"))
    run_gpu_ranks(1, _single_rank, d)
    return d, torch.load(os.path.join(d, "single.pt"))


@pytest.mark.parametrize("name", list(LAYOUTS))
def test_layout_matches_one_gpu(name, single):
    from nano_megatron_b200.utils.sharding import merge_shards

    layout, world = LAYOUTS[name]
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    d, ref = single
    run_gpu_ranks(world, _layout_rank, layout, d)
    results = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(world)]
    for r in results:
        assert abs(r["loss"] - ref["loss"]) < 2e-2 * abs(ref["loss"]), (name, r["loss"])
    by_tp: dict[int, dict] = {}
    for r in results:
        if r["dp_rank"] == 0:
            by_tp.setdefault(r["tp_rank"], {}).update(r["grads"])
    tp = results[0]["tp"]
    merged = merge_shards([by_tp[i] for i in range(tp)]) if tp > 1 else by_tp[0]
    ref_grads = ref["grads"]
    if "lm_head.weight" in merged and "lm_head.weight" not in ref_grads:
        tied = merged.pop("lm_head.weight")
        e = ref_grads["embedding.weight"]
        assert ((tied - e).norm() / e.norm()).item() < 5e-2
    assert set(merged) == set(ref_grads), set(ref_grads) ^ set(merged)
    for k, g in ref_grads.items():
        err = ((merged[k] - g).norm() / (g.norm() + 1e-12)).item()
        assert err < 5e-2, f"{name}: {k} rel err {err}"
