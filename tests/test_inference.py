"""Checkpoint export -> single-device artifact -> generation (CPU, gloo).

Reference counterparts: tests/integration/test_inference_export.py and
tests/unit/test_generation.py. The KV-cached decoder must pick exactly the
tokens the full-prefix recompute picks; a TP2xPP2 checkpoint must export to the
same weights as the single-process model it was sharded from; and the
reference's own exporter (when installed) must accept our checkpoints.
"""

from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from dist_utils import run_ranks

TEXTS = ["once upon a time there was a little cat who liked to run in the sun. "
         "the cat saw a dog and they played all day." * 2,
         "a girl named lily found a red ball in the park and was very happy."] * 20


def _tokenizer(root: Path):
    from nano_megatron_b200.tokenizer import ByteBPETrainingConfig, ByteLevelBPETokenizer

    d = root / "tok"
    if not (root / "train.jsonl").exists():
        (root / "train.jsonl").write_text("".join(json.dumps({"text": t}) + "\n" for t in TEXTS))
    if not d.exists():
        ByteLevelBPETokenizer.train(TEXTS, ByteBPETrainingConfig(vocab_size=320)).save(d)
    return ByteLevelBPETokenizer.load(d), d


def _cfg(root: Path, vocab: int, *, tp=1, pp=1, dp=1, mode="ddp"):
    from nano_megatron_b200.config import config_from_dict

    return config_from_dict({
        "data_parallel": {"mode": mode},
        "model": {"layers": 4, "hidden_size": 64, "ffn_hidden_size": 128, "heads": 4,
                  "kv_heads": 2, "seq_length": 64, "vocab_size": vocab},
        "parallel": {"tensor": tp, "pipeline": pp, "context": 1, "expert": 1, "data": dp,
                     "sequence_parallel": False},
        "precision": {"params": "float32", "compute": "float32"},
        "distributed": {"device": "cpu", "backend": "gloo"},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 2},
        "optimizer": {"lr": 1e-2},
        "data": {"text_path": str(root / "train.jsonl"), "tokenizer": {"path": str(root / "tok")}},
        "checkpoint": {"directory": str(root / "ck")}})


def _train_and_save(cfg, steps=2, weights=None):
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    torch.manual_seed(0)
    rt = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, rt)
    if weights is not None:
        _load_global(comps, weights)
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    return comps, tr


def _load_global(comps, full):
    import re

    from nano_megatron_b200.utils.sharding import shard_tensor, tensor_shard_dim

    parts = getattr(comps.built, "partitions", None) or (comps.built.partition,)
    tp = comps.parallel.tp
    with torch.no_grad():
        for name, p in comps.model.named_parameters():
            m = re.match(r"(?:chunks\.(\d+)\.)?model\.(.*)$", name)
            rest = m.group(2)
            lm = re.match(r"layers\.(\d+)\.(.*)$", rest)
            if lm:
                rest = f"layers.{parts[int(m.group(1) or 0)].start_layer + int(lm.group(1))}." \
                       f"{lm.group(2)}"
            p.copy_(shard_tensor(full[rest], tensor_shard_dim(rest), tp.rank, tp.size))


def test_export_and_kv_cache_generation(tmp_path):
    from nano_megatron_b200.inference import (export_checkpoint, generate_from_artifact,
                                              load_inference_artifact)

    tok, _ = _tokenizer(tmp_path)
    cfg = _cfg(tmp_path, tok.vocab_size)
    comps, tr = _train_and_save(cfg)
    ids = torch.tensor([tok.encode(TEXTS[0])[:65]] * 4)
    tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    path = tr.save_checkpoint()
    art = export_checkpoint(path, tmp_path / "artifact")
    assert (tmp_path / "artifact" / ".complete").is_file()
    man = json.loads((tmp_path / "artifact" / "manifest.json").read_text())
    assert man["artifact"] == "nano_megatron.single_device_gpt" and man["format_version"] == 1
    live = {k.removeprefix("model."): v for k, v in comps.model.state_dict().items()}
    for k, v in art.state_dict.items():
        torch.testing.assert_close(v, live[k], rtol=0, atol=0)
    assert load_inference_artifact(tmp_path / "artifact").weight_dtype == torch.float32
    with pytest.raises(FileExistsError):
        export_checkpoint(path, tmp_path / "artifact")
    for temp, k, p in ((0.0, 0, 1.0), (0.9, 20, 0.9)):
        a = generate_from_artifact(tmp_path / "artifact", "once upon", device="cpu",
                                   max_new_tokens=24, temperature=temp, top_k=k, top_p=p,
                                   seed=7, use_kv_cache=True)
        b = generate_from_artifact(tmp_path / "artifact", "once upon", device="cpu",
                                   max_new_tokens=24, temperature=temp, top_k=k, top_p=p,
                                   seed=7, use_kv_cache=False)
        assert a.generated_token_ids == b.generated_token_ids
        assert a.text.startswith("once upon")
    with pytest.raises(ValueError, match="exceeds model sequence length"):
        generate_from_artifact(tmp_path / "artifact", "once", device="cpu", max_new_tokens=64)


def _sharded_save(rank, world, root, weights_path):
    root = Path(root)
    tok, _ = _tokenizer(root)
    cfg = _cfg(root, tok.vocab_size, tp=2, pp=2)
    comps, tr = _train_and_save(cfg, weights=torch.load(weights_path))
    tr.save_checkpoint()


@pytest.mark.distributed
def test_tp2_pp2_checkpoint_exports_global_weights(tmp_path):
    from nano_megatron_b200.inference import export_checkpoint

    tok, _ = _tokenizer(tmp_path)
    cfg = _cfg(tmp_path, tok.vocab_size)
    comps, _ = _train_and_save(cfg)
    full = {k.removeprefix("model."): v.clone() for k, v in comps.model.state_dict().items()}
    wp = tmp_path / "full.pt"
    torch.save(full, wp)
    run_ranks(4, _sharded_save, str(tmp_path), str(wp))
    ck = sorted((tmp_path / "ck").glob("step_*"))[-1]
    art = export_checkpoint(ck, tmp_path / "artifact_tp2pp2")
    assert art.manifest["source"]["parallel_sizes"]["tp"] == 2
    for k, v in full.items():
        torch.testing.assert_close(art.state_dict[k], v, rtol=0, atol=0)
    if importlib.util.find_spec("nano_megatron") is not None or \
            (Path(__file__).parents[1] / "baseline" / "_ref" / "nano_megatron").is_dir():
        env = dict(os.environ, PYTHONPATH=str(Path(__file__).parents[1] / "baseline" / "_ref"))
        code = ("import sys; from nano_megatron.inference import export_checkpoint as e; "
                "a = e(sys.argv[1], sys.argv[2]); print(len(a.state_dict))")
        r = subprocess.run([sys.executable, "-c", code, str(ck), str(tmp_path / "ref_art")],
                           env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        ref = torch.load(tmp_path / "ref_art" / "model.pt")
        for k, v in full.items():
            torch.testing.assert_close(ref[k], v, rtol=0, atol=0)


def _zero3_save(rank, world, root, weights_path):
    root = Path(root)
    tok, _ = _tokenizer(root)
    cfg = _cfg(root, tok.vocab_size, tp=2, dp=2, mode="zero3")
    from nano_megatron_b200.checkpoint import CheckpointManager
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    comps = build_training_components(cfg, DistributedRuntime(cfg.distributed).initialize())
    ck = CheckpointManager(config=cfg.checkpoint, parallel=comps.parallel, run_config=cfg)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, checkpoint=ck, rng=comps.rng)
    with comps.data_parallel.full_parameters():
        _load_global(comps, torch.load(weights_path))
    comps.data_parallel.load_model_parameters()
    tr.save_checkpoint()


@pytest.mark.distributed
def test_zero3_tp2_checkpoint_exports_global_weights(tmp_path):
    """A TP2 x DP2 ZeRO-3 checkpoint (FSDP2 DCP layout) exports to the global weights."""
    from nano_megatron_b200.checkpoint.manifest import CheckpointManifest
    from nano_megatron_b200.inference import export_checkpoint

    tok, _ = _tokenizer(tmp_path)
    comps, _ = _train_and_save(_cfg(tmp_path, tok.vocab_size))
    full = {k.removeprefix("model."): v.clone() for k, v in comps.model.state_dict().items()}
    wp = tmp_path / "full.pt"
    torch.save(full, wp)
    run_ranks(4, _zero3_save, str(tmp_path), str(wp))
    ck = sorted((tmp_path / "ck").glob("step_*"))[-1]
    assert CheckpointManifest.read(ck / "manifest.json").storage_backend == "fsdp2_dcp"
    art = export_checkpoint(ck, tmp_path / "artifact_zero3")
    for k, v in full.items():
        torch.testing.assert_close(art.state_dict[k], v, rtol=0, atol=0)
