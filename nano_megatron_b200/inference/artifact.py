"""Single-device GPT artifacts exported from training checkpoints.

An artifact directory holds ``model.pt`` (the merged, unsharded state dict with
the single-device GPT key names), ``tokenizer/`` (a byte-level BPE artifact),
``manifest.json`` (artifact ``nano_megatron.single_device_gpt`` version 1: model
config, source checkpoint, tokenizer identity, weight dtype/sha256/count) and a
``.complete`` marker; it is assembled in a temporary sibling directory,
re-validated, then renamed into place. The artifact format, its manifest
fields and its validation rules follow the reference
(src/nano_megatron/inference/artifact.py:31-742) so artifacts are
interchangeable in both directions.

Merging: every rank-local shard's tensors are placed into their global tensor
at the offsets recorded in the shard metadata (tensor-parallel pieces must tile
the global tensor exactly; replicated copies must agree bit for bit), and
pipeline-local layer indices are mapped back to global ones through each
shard's layer ranges. Unlike the reference this also exports interleaved
(virtual-stage) pipeline checkpoints, whose keys are ``chunks.<c>.model.*``,
and ZeRO-3 checkpoints, whose rank-local states are already logical tensors.
"""

from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import tempfile
from collections.abc import Mapping
from dataclasses import dataclass, fields
from pathlib import Path
from types import SimpleNamespace
from typing import Any

import torch

from nano_megatron_b200.checkpoint import CheckpointManifest, ShardMetadata
from nano_megatron_b200.config import GPTConfig, TrainConfig, config_from_dict, load_config
from nano_megatron_b200.config.validation import validate_config
from nano_megatron_b200.parallel.axes import ParallelAxis
from nano_megatron_b200.tokenizer import ByteLevelBPETokenizer, validate_tokenizer_for_model

ARTIFACT_NAME = "nano_megatron.single_device_gpt"
ARTIFACT_VERSION = 1
MANIFEST_FILE = "manifest.json"
MODEL_FILE = "model.pt"
TOKENIZER_DIR = "tokenizer"
COMPLETE_FILE = ".complete"
DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
_KEY = re.compile(r"^(?:chunks\.(\d+)\.)?model\.(.+)$")
_LAYER = re.compile(r"^layers\.(\d+)\.(.+)$")


class InferenceArtifactError(ValueError):
    """A checkpoint or an exported artifact violates its contract."""


@dataclass(frozen=True, slots=True)
class InferenceArtifact:
    path: Path
    manifest: dict[str, Any]
    model_config: GPTConfig
    tokenizer: ByteLevelBPETokenizer
    state_dict: dict[str, torch.Tensor]
    weight_dtype: torch.dtype


def local_parallel():
    """A one-rank stand-in for the parallel state (TP=PP=CP=1)."""
    g = SimpleNamespace(rank=0, size=1, process_group=None, ranks=(0,))
    return SimpleNamespace(tp=g, pp=g, cp=g, ep=g, dp=g, sequence_parallel=False)


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _json(path: Path, what: str) -> dict:
    try:
        v = json.loads(Path(path).read_text(encoding="utf-8"))
    except (OSError, UnicodeError, ValueError) as e:
        raise InferenceArtifactError(f"could not read {what} {path}: {e}") from e
    if not isinstance(v, dict):
        raise InferenceArtifactError(f"{what} must contain a JSON object: {path}")
    return v


def _inside(root: Path, rel: str, what: str) -> Path:
    p = Path(rel)
    if p.is_absolute() or ".." in p.parts:
        raise InferenceArtifactError(f"invalid {what} path: {rel!r}")
    if not (root / p).is_file():
        raise FileNotFoundError(f"{what} does not exist: {root / p}")
    return root / p


def _load_mapping(path: Path, what: str) -> Mapping:
    try:
        v = torch.load(path, map_location="cpu", weights_only=True)
    except (OSError, RuntimeError, ValueError) as e:
        raise InferenceArtifactError(f"could not load {what} {path}: {e}") from e
    if not isinstance(v, Mapping):
        raise InferenceArtifactError(f"{what} must contain a mapping: {path}")
    return v


def model_config_dict(cfg: GPTConfig) -> dict[str, Any]:
    return {f.name: getattr(cfg, f.name) for f in fields(GPTConfig)}


def parse_model_config(v: Any) -> GPTConfig:
    if not isinstance(v, Mapping):
        raise InferenceArtifactError("artifact model config must be an object")
    names = {f.name for f in fields(GPTConfig)}
    missing, unknown = names - set(v), set(v) - names
    if missing or unknown:
        parts = (["missing " + ", ".join(sorted(missing))] if missing else []) + \
            (["unknown " + ", ".join(sorted(unknown))] if unknown else [])
        raise InferenceArtifactError("invalid artifact model config (" + "; ".join(parts) + ")")
    try:
        return GPTConfig(**{n: v[n] for n in names})
    except (TypeError, ValueError) as e:
        raise InferenceArtifactError(f"invalid artifact model config: {e}") from e


def expected_shapes(cfg: GPTConfig) -> dict[str, tuple[int, ...]]:
    from nano_megatron_b200.models.gpt.model import GPTModel

    with torch.device("meta"):
        m = GPTModel(cfg, parallel=local_parallel())
    return {k: tuple(t.shape) for k, t in m.state_dict().items()}


def _world(manifest: CheckpointManifest) -> int:
    n = 1
    for axis in ("tp", "pp", "cp", "ep", "dp"):
        if axis not in manifest.parallel_sizes:
            raise InferenceArtifactError(f"checkpoint manifest is missing parallel size {axis!r}")
        s = int(manifest.parallel_sizes[axis])
        if s < 1:
            raise InferenceArtifactError(f"invalid parallel sizes {manifest.parallel_sizes}")
        n *= s
    return n


def _train_config(manifest: CheckpointManifest, config_path: Path | None) -> TrainConfig:
    embedded = None
    if isinstance(manifest.run_config, Mapping):
        try:
            embedded = config_from_dict(manifest.run_config)
        except (TypeError, ValueError) as e:
            if config_path is None:
                raise InferenceArtifactError(f"checkpoint run_config cannot be reconstructed: "
                                             f"{e}") from e
    if config_path is None:
        if embedded is None:
            raise InferenceArtifactError("checkpoint has no usable run_config; pass --config "
                                         "explicitly")
        cfg = embedded
    else:
        cfg = load_config(config_path, world_size=_world(manifest), emit_warnings=False)
        if embedded is not None and cfg.model != embedded.model:
            raise InferenceArtifactError("explicit config model does not match checkpoint "
                                         "run_config model")
    validate_config(cfg, world_size=_world(manifest))
    want = {"tp": cfg.parallel.tensor, "pp": cfg.parallel.pipeline, "cp": cfg.parallel.context,
            "ep": cfg.parallel.expert}
    if cfg.parallel.data is not None:
        want["dp"] = cfg.parallel.data
    bad = {a: (manifest.parallel_sizes.get(a), w) for a, w in want.items()
           if manifest.parallel_sizes.get(a) != w}
    if bad:
        raise InferenceArtifactError(f"config parallel sizes do not match checkpoint manifest: "
                                     f"{bad}")
    if cfg.pipeline.virtual_stages_per_rank != manifest.virtual_stages_per_rank:
        raise InferenceArtifactError(
            "config virtual pipeline size does not match checkpoint manifest: "
            f"{cfg.pipeline.virtual_stages_per_rank} != {manifest.virtual_stages_per_rank}")
    return cfg


def _source_tokenizer(cfg: TrainConfig, override: Path | None):
    src = override
    if src is None:
        tok = cfg.data.tokenizer
        if tok is None and cfg.validation.data is not None:
            tok = cfg.validation.data.tokenizer
        src = None if tok is None else Path(tok.path)
    if src is None:
        raise InferenceArtifactError("checkpoint config has no tokenizer; pass --tokenizer "
                                     "explicitly")
    try:
        tokenizer = ByteLevelBPETokenizer.load(src)
    except (FileNotFoundError, NotADirectoryError, ValueError) as e:
        if override is None:
            raise InferenceArtifactError(f"could not load checkpoint tokenizer {src}; pass "
                                         f"--tokenizer to override: {e}") from e
        raise
    validate_tokenizer_for_model(tokenizer, cfg.model)
    return tokenizer, src


# ---------------------------------------------------------------------- merge
class _Assembler:
    """Collects shard pieces into global tensors and checks exact coverage."""

    def __init__(self) -> None:
        self.full: dict[str, torch.Tensor] = {}
        self.sharded: dict[str, bool] = {}
        self.covered: dict[str, torch.Tensor] = {}

    def add(self, key: str, t: torch.Tensor, meta: ShardMetadata) -> None:
        if tuple(t.shape) != tuple(meta.local_shape):
            raise InferenceArtifactError(f"checkpoint tensor {key!r} shape {tuple(t.shape)} does "
                                         f"not match metadata {meta.local_shape}")
        if any(a is not ParallelAxis.TP for a in meta.sharded_axes):
            raise InferenceArtifactError(f"checkpoint tensor {key!r} uses unsupported sharding "
                                         f"axes {[a.value for a in meta.sharded_axes]}")
        sharded = ParallelAxis.TP in meta.sharded_axes
        if key in self.sharded and self.sharded[key] != sharded:
            raise InferenceArtifactError(f"checkpoint tensor {key!r} mixes sharded and "
                                         "replicated pieces")
        t = t.detach().cpu()
        if not sharded:
            if tuple(meta.local_shape) != tuple(meta.global_shape) or any(meta.global_offset):
                raise InferenceArtifactError(f"replicated checkpoint tensor {key!r} has "
                                             "non-replicated metadata")
            prev = self.full.get(key)
            if prev is None:
                self.full[key], self.sharded[key] = t.clone(), False
            elif prev.dtype != t.dtype or not torch.equal(prev, t):
                raise InferenceArtifactError(f"replicated TP copies differ for checkpoint tensor "
                                             f"{key!r}")
            return
        g = self.full.get(key)
        if g is None:
            g = self.full[key] = torch.empty(tuple(meta.global_shape), dtype=t.dtype)
            self.covered[key] = torch.zeros(tuple(meta.global_shape), dtype=torch.uint8)
            self.sharded[key] = True
        if tuple(g.shape) != tuple(meta.global_shape) or g.dtype != t.dtype:
            raise InferenceArtifactError(f"checkpoint tensor {key!r} has inconsistent global "
                                         "shape or dtype")
        box = tuple(slice(o, o + s) for o, s in zip(meta.global_offset, meta.local_shape))
        if self.covered[key][box].any():
            raise InferenceArtifactError(f"checkpoint tensor {key!r} has overlapping TP shards")
        g[box].copy_(t)
        self.covered[key][box] = 1

    def finish(self, cfg: GPTConfig) -> dict[str, torch.Tensor]:
        for k, cov in self.covered.items():
            if not bool(cov.all()):
                raise InferenceArtifactError(f"checkpoint tensor {k!r} TP shards cover "
                                             f"{int(cov.sum())} of {cov.numel()} elements")
        state = dict(self.full)
        exp = expected_shapes(cfg)
        missing, extra = set(exp) - set(state), set(state) - set(exp)
        if missing or extra:
            parts = (["missing " + ", ".join(sorted(missing))] if missing else []) + \
                (["unexpected " + ", ".join(sorted(extra))] if extra else [])
            raise InferenceArtifactError("merged model state keys are invalid (" +
                                         "; ".join(parts) + ")")
        for k, s in exp.items():
            if tuple(state[k].shape) != s:
                raise InferenceArtifactError(f"merged tensor {k!r} shape "
                                             f"{tuple(state[k].shape)} != {s}")
        if cfg.tie_embeddings:
            if not torch.equal(state["embedding.weight"], state["lm_head.weight"]):
                raise InferenceArtifactError("checkpoint tied embedding and LM-head weights are "
                                             "not synchronized")
            state["lm_head.weight"] = state["embedding.weight"]
        return state


def _global_key(key: str, ranges) -> str:
    m = _KEY.fullmatch(key)
    if m is None:
        raise InferenceArtifactError(f"checkpoint model key does not use the GPT pipeline "
                                     f"wrapper prefix: {key!r}")
    chunk, rest = int(m.group(1) or 0), m.group(2)
    lm = _LAYER.fullmatch(rest)
    if lm is None or ranges is None:
        return rest
    if chunk >= len(ranges):
        raise InferenceArtifactError(f"checkpoint key {key!r} names virtual stage {chunk} with "
                                     "no layer range")
    start, end = ranges[chunk]
    local = int(lm.group(1))
    if not 0 <= local < end - start:
        raise InferenceArtifactError(f"checkpoint layer key {key!r} is outside shard layer "
                                     f"range [{start}, {end})")
    return f"layers.{start + local}.{lm.group(2)}"


def _shard_ranges(shard):
    if shard.layer_ranges:
        return tuple(tuple(r) for r in shard.layer_ranges)
    if shard.layer_start is None or shard.layer_end is None:
        raise InferenceArtifactError(f"shard {shard.shard_id} has no pipeline layer range "
                                     "metadata")
    return ((shard.layer_start, shard.layer_end),)


def merge_checkpoint_model(checkpoint: Path, manifest: CheckpointManifest,
                           cfg: GPTConfig) -> dict[str, torch.Tensor]:
    asm = _Assembler()
    if manifest.storage_backend == "torch.save":
        if any(manifest.parallel_sizes.get(a, 1) != 1 for a in ("tp", "pp", "ep")):
            raise InferenceArtifactError("torch.save checkpoint without rank-local shards must "
                                         "have TP=PP=EP=1")
        payload = _load_mapping(checkpoint / MODEL_FILE, "checkpoint model state")
        if set(payload) != set(manifest.tensor_metadata):
            raise InferenceArtifactError("checkpoint model keys do not match manifest metadata")
        for k, t in payload.items():
            if not isinstance(k, str) or not isinstance(t, torch.Tensor):
                raise InferenceArtifactError("checkpoint model state must contain string Tensor "
                                             "entries")
            asm.add(_global_key(k, None), t, manifest.tensor_metadata[k])
        return asm.finish(cfg)
    if manifest.storage_backend not in ("rank_local_torch.save", "fsdp2_dcp"):
        raise InferenceArtifactError(f"checkpoint backend {manifest.storage_backend!r} cannot "
                                     "be exported; supported backends are "
                                     "rank_local_torch.save, fsdp2_dcp and torch.save")
    if manifest.parallel_sizes.get("ep", 1) != 1:
        raise InferenceArtifactError("checkpoint export currently requires EP=1")
    tp, pp = manifest.parallel_sizes["tp"], manifest.parallel_sizes["pp"]
    if manifest.storage_backend == "fsdp2_dcp":
        return _merge_zero3(checkpoint, manifest, cfg, tp, pp, asm)
    shards = [s for s in manifest.rank_local_shards if s.ep == 0]
    coords = {(s.tp, s.pp) for s in shards}
    if len(shards) != tp * pp or coords != {(t, p) for t in range(tp) for p in range(pp)}:
        raise InferenceArtifactError(f"checkpoint TP/PP shard coordinates are incomplete: "
                                     f"{sorted(coords)}")
    for s in sorted(shards, key=lambda s: (s.pp, s.tp)):
        path = _inside(checkpoint, s.state_file, "rank-local checkpoint state")
        model = _load_mapping(path, "rank-local checkpoint state").get("model")
        if not isinstance(model, Mapping):
            raise InferenceArtifactError(f"rank-local checkpoint state {path} has no model")
        if set(model) != set(s.tensor_metadata):
            raise InferenceArtifactError(f"rank-local state keys do not match manifest metadata: "
                                         f"{path}")
        ranges = _shard_ranges(s) if pp > 1 or manifest.virtual_stages_per_rank > 1 else None
        for k, t in model.items():
            if not isinstance(k, str) or not isinstance(t, torch.Tensor):
                raise InferenceArtifactError(f"rank-local model state must contain string Tensor "
                                             f"entries: {path}")
            asm.add(_global_key(k, ranges), t, s.tensor_metadata[k])
    return asm.finish(cfg)


def _merge_zero3(checkpoint: Path, manifest: CheckpointManifest, cfg: GPTConfig, tp: int,
                 pp: int, asm) -> dict[str, torch.Tensor]:
    """ZeRO-3 checkpoints: one DCP directory per (tp, pp) coordinate; the shard description
    written beside it gives the TP shard metadata and layer ranges."""
    from nano_megatron_b200.checkpoint.fsdp2_format import (SHARD_INFO_FILE, load_dcp_model,
                                                           zero3_state_dir)
    from nano_megatron_b200.checkpoint.manifest import RankLocalShard

    for p_ in range(pp):
        for t_ in range(tp):
            d = zero3_state_dir(checkpoint, t_, p_)
            info_path = d / SHARD_INFO_FILE
            if not info_path.is_file():
                raise InferenceArtifactError(
                    f"ZeRO-3 checkpoint directory {d} has no {SHARD_INFO_FILE} shard description "
                    "(written by this framework); cannot place its tensors")
            shard = RankLocalShard.from_dict(json.loads(info_path.read_text()))
            model = load_dcp_model(d)
            if set(model) != set(shard.tensor_metadata):
                raise InferenceArtifactError(f"ZeRO-3 model keys do not match the shard "
                                             f"description: {d}")
            ranges = _shard_ranges(shard) if pp > 1 or manifest.virtual_stages_per_rank > 1 \
                else None
            for k, t in model.items():
                asm.add(_global_key(k, ranges), t, shard.tensor_metadata[k])
    return asm.finish(cfg)


# ---------------------------------------------------------------------- export / load
def _check_target(d: Path) -> bool:
    if d.is_symlink():
        raise FileExistsError(f"refusing to replace inference artifact symlink: {d}")
    if not d.exists():
        return False
    if not d.is_dir():
        raise FileExistsError(f"inference artifact path already exists: {d}")
    if any(d.iterdir()):
        raise FileExistsError(f"refusing to overwrite non-empty inference artifact directory: "
                              f"{d}")
    return True


def export_checkpoint(checkpoint_path, output_path, *, config_path=None,
                      tokenizer_path=None) -> InferenceArtifact:
    """Merge one training checkpoint into an atomically published single-device artifact."""
    ck = Path(checkpoint_path)
    if not ck.is_dir() or not (ck / COMPLETE_FILE).is_file():
        raise ValueError(f"checkpoint is incomplete or missing: {ck}")
    man_path = ck / MANIFEST_FILE
    manifest = CheckpointManifest.read(man_path)
    if manifest.framework != "nano-megatron":
        raise InferenceArtifactError(f"unsupported checkpoint framework: {manifest.framework!r}")
    cfg = _train_config(manifest, None if config_path is None else Path(config_path))
    tokenizer, tok_src = _source_tokenizer(cfg, None if tokenizer_path is None
                                           else Path(tokenizer_path))
    state = merge_checkpoint_model(ck, manifest, cfg.model)
    dtypes = {t.dtype for t in state.values() if t.is_floating_point()}
    if len(dtypes) != 1:
        raise InferenceArtifactError(f"exported GPT weights must use exactly one floating dtype, "
                                     f"got {dtypes}")
    wdtype = next(iter(dtypes))
    names = {v: k for k, v in DTYPES.items()}
    if wdtype not in names:
        raise InferenceArtifactError(f"unsupported model weight dtype: {wdtype}")
    dest = Path(output_path)
    was_empty = _check_target(dest)
    dest.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=f".{dest.name}.tmp-", dir=dest.parent))
    removed = False
    try:
        torch.save(state, tmp / MODEL_FILE)
        tokenizer.save(tmp / TOKENIZER_DIR)
        manifest_out = {
            "artifact": ARTIFACT_NAME, "format_version": ARTIFACT_VERSION,
            "framework": "nano-megatron", "model": model_config_dict(cfg.model),
            "source": {"checkpoint": str(ck.resolve()),
                       "checkpoint_manifest_sha256": sha256_file(man_path),
                       "data_parallel_mode": manifest.data_parallel_mode,
                       "parallel_sizes": dict(manifest.parallel_sizes), "step": manifest.step,
                       "storage_backend": manifest.storage_backend},
            "tokenizer": {"directory": TOKENIZER_DIR, "eos_token_id": tokenizer.eos_token_id,
                          "fingerprint": tokenizer.fingerprint,
                          "source": str(Path(tok_src).resolve()),
                          "vocab_size": tokenizer.vocab_size},
            "weights": {"dtype": names[wdtype], "file": MODEL_FILE,
                        "sha256": sha256_file(tmp / MODEL_FILE), "tensors": len(state)}}
        (tmp / MANIFEST_FILE).write_text(json.dumps(manifest_out, ensure_ascii=False, indent=2,
                                                    sort_keys=True) + "\n", encoding="utf-8")
        (tmp / COMPLETE_FILE).write_text("complete\n", encoding="utf-8")
        del state
        load_inference_artifact(tmp)
        if was_empty:
            dest.rmdir()
            removed = True
        elif dest.exists() or dest.is_symlink():
            raise FileExistsError(f"inference artifact path already exists: {dest}")
        os.replace(tmp, dest)
    except BaseException:
        if removed and not dest.exists():
            dest.mkdir()
        raise
    finally:
        if tmp.exists():
            shutil.rmtree(tmp)
    return load_inference_artifact(dest)


def load_inference_artifact(path) -> InferenceArtifact:
    """Load and fully validate one exported single-device artifact on CPU."""
    d = Path(path)
    if not d.is_dir() or not (d / COMPLETE_FILE).is_file():
        raise ValueError(f"inference artifact is incomplete or missing: {d}")
    man = _json(d / MANIFEST_FILE, "inference manifest")
    if man.get("artifact") != ARTIFACT_NAME:
        raise InferenceArtifactError(f"unsupported inference artifact: {man.get('artifact')!r}")
    if man.get("format_version") != ARTIFACT_VERSION:
        raise InferenceArtifactError(f"unsupported inference artifact version: "
                                     f"{man.get('format_version')!r}")
    cfg = parse_model_config(man.get("model"))
    tinfo = man.get("tokenizer")
    if not isinstance(tinfo, Mapping) or not isinstance(tinfo.get("directory"), str):
        raise InferenceArtifactError("inference manifest tokenizer must be an object with a "
                                     "string directory")
    trel = Path(tinfo["directory"])
    if trel.is_absolute() or ".." in trel.parts:
        raise InferenceArtifactError("inference tokenizer directory must be relative")
    tokenizer = ByteLevelBPETokenizer.load(d / trel)
    validate_tokenizer_for_model(tokenizer, cfg)
    for field, actual in (("fingerprint", tokenizer.fingerprint),
                          ("vocab_size", tokenizer.vocab_size),
                          ("eos_token_id", tokenizer.eos_token_id)):
        if tinfo.get(field) != actual:
            raise InferenceArtifactError(f"inference tokenizer {field} does not match manifest")
    winfo = man.get("weights")
    if not isinstance(winfo, Mapping) or not isinstance(winfo.get("file"), str):
        raise InferenceArtifactError("inference manifest weights must be an object with a "
                                     "string file")
    wpath = _inside(d, winfo["file"], "inference weights")
    if not isinstance(winfo.get("sha256"), str) or sha256_file(wpath) != winfo["sha256"]:
        raise InferenceArtifactError("inference weights SHA256 does not match manifest")
    if winfo.get("dtype") not in DTYPES:
        raise InferenceArtifactError(f"unsupported inference weight dtype: "
                                     f"{winfo.get('dtype')!r}")
    wdtype = DTYPES[winfo["dtype"]]
    state: dict[str, torch.Tensor] = {}
    for k, v in _load_mapping(wpath, "inference weights").items():
        if not isinstance(k, str) or not isinstance(v, torch.Tensor):
            raise InferenceArtifactError("inference weights must contain only string Tensor "
                                         "entries")
        if v.is_floating_point() and v.dtype is not wdtype:
            raise InferenceArtifactError(f"inference tensor {k!r} dtype {v.dtype} != {wdtype}")
        state[k] = v
    if winfo.get("tensors") != len(state):
        raise InferenceArtifactError("inference weights tensor count does not match manifest")
    exp = expected_shapes(cfg)
    if set(state) != set(exp):
        raise InferenceArtifactError("inference weight keys do not match GPT model state")
    for k, s in exp.items():
        if tuple(state[k].shape) != s:
            raise InferenceArtifactError(f"inference tensor {k!r} shape {tuple(state[k].shape)} "
                                         f"!= {s}")
    if cfg.tie_embeddings:
        if not torch.equal(state["embedding.weight"], state["lm_head.weight"]):
            raise InferenceArtifactError("inference tied embedding weights differ")
        state["lm_head.weight"] = state["embedding.weight"]
    return InferenceArtifact(d.resolve(), man, cfg, tokenizer, state, wdtype)
