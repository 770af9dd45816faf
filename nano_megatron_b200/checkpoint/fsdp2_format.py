"""ZeRO-3 checkpoints in the reference's FSDP2 distributed-checkpoint layout.

The reference saves ZeRO-3 state as one torch.distributed.checkpoint (DCP) directory per
(domain, tp, pp) coordinate, ``fsdp2_states/dense_tpXXXX_ppXXXX``, holding
``{"model": model_state, "optimizer": optimizer_state}`` as produced by
``torch.distributed.checkpoint.state_dict.get_state_dict`` on its FSDP2 module
(src/nano_megatron/checkpoint/manager.py:733-786, src/nano_megatron/data_parallel/zero3.py:256-291):

* ``model``: the stage's state dict by fully-qualified name (a tied LM head appears under
  both names);
* ``optimizer``: ``{"state": {fqn: {"exp_avg", "exp_avg_sq", "step"}}, "param_groups":
  [torch AdamW's group with "params" = the parameter FQNs]}``, one entry per distinct
  parameter.

Our ZeRO-3 keeps flat fp32 shards per bucket instead of FSDP2 DTensors; this module maps
between the two. Writing uses one DCP writer per coordinate with whole tensors (DCP
reshards them when the reference loads onto its DP mesh); reading loads whole tensors.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any, Mapping

import torch


# Our description of the coordinate's shard (layer ranges, TP shard metadata), written next
# to the DCP files so that ZeRO-3 checkpoints can be exported; DCP readers ignore it.
SHARD_INFO_FILE = "nmb_shard.json"


def zero3_state_dir(root: Path, tp: int, pp: int) -> Path:
    return Path(root) / "fsdp2_states" / f"dense_tp{tp:04d}_pp{pp:04d}"


def _adamw_group(lr: float, betas, eps: float, weight_decay: float) -> dict:
    """torch AdamW's parameter-group fields (the same keys a freshly built AdamW has)."""
    probe = torch.optim.AdamW([torch.nn.Parameter(torch.zeros(1))], lr=float(lr),
                              betas=tuple(float(b) for b in betas), eps=float(eps),
                              weight_decay=float(weight_decay))
    group = dict(probe.param_groups[0])
    group.pop("params")
    return group


def to_fsdp2_state(model_state: Mapping[str, torch.Tensor], dp_state: Mapping[str, Any],
                   buckets, *, betas, eps: float, weight_decay: float) -> dict:
    """Build the nested DCP state from a model state dict and our ZeRO bucket state.

    ``dp_state`` is the strategy's logical state (``{"step", "learning_rate", "buckets":
    {index: {"exp_avg", "exp_avg_sq", ...}}}`` with whole-bucket tensors); ``buckets`` gives
    each bucket's parameter slices (name, start, end, shape)."""
    step = torch.tensor(float(dp_state["step"]), dtype=torch.float32)
    state: dict[str, dict[str, torch.Tensor]] = {}
    order: list[str] = []
    for b in buckets:
        entry = dp_state["buckets"].get(str(b.index), dp_state["buckets"].get(b.index))
        for s in b.slices:
            shape = tuple(model_state[s.name].shape)
            state[s.name] = {
                "exp_avg": entry["exp_avg"][s.start:s.end].reshape(shape).clone(),
                "exp_avg_sq": entry["exp_avg_sq"][s.start:s.end].reshape(shape).clone(),
                "step": step.clone(),
            }
            order.append(s.name)
    # The reference's optimizer lists parameters in module order; keep ours in the order
    # of the model state dict (the same module order), skipping tied duplicates.
    ranked = [k for k in model_state if k in state]
    ranked += [k for k in order if k not in set(ranked)]
    group = _adamw_group(dp_state["learning_rate"], betas, eps, weight_decay)
    group["params"] = ranked
    return {"model": {k: v for k, v in model_state.items()},
            "optimizer": {"state": {k: state[k] for k in ranked}, "param_groups": [group]}}


def from_fsdp2_state(nested: Mapping[str, Any], buckets, mode: str = "zero3") -> dict:
    """Our ZeRO bucket state from a loaded FSDP2 DCP state (whole tensors, any rank)."""
    model = nested["model"]
    optim = nested["optimizer"]
    per_param = optim["state"]
    groups = optim.get("param_groups") or [{}]
    steps = {int(round(float(v["step"]))) for v in per_param.values() if "step" in v}
    if len(steps) > 1:
        raise ValueError(f"inconsistent optimizer steps in the ZeRO-3 checkpoint: {steps}")
    out_buckets: dict[str, dict] = {}
    for b in buckets:
        fields = {"master_parameter": [], "exp_avg": [], "exp_avg_sq": []}
        for s in b.slices:
            if s.name not in model:
                raise KeyError(f"parameter {s.name!r} missing from the ZeRO-3 checkpoint")
            fields["master_parameter"].append(model[s.name].reshape(-1).float())
            st = per_param.get(s.name)
            if st is None:   # never stepped: zero moments, as a fresh AdamW would have
                zeros = torch.zeros(s.end - s.start, dtype=torch.float32)
                fields["exp_avg"].append(zeros)
                fields["exp_avg_sq"].append(zeros.clone())
            else:
                fields["exp_avg"].append(st["exp_avg"].reshape(-1).float())
                fields["exp_avg_sq"].append(st["exp_avg_sq"].reshape(-1).float())
        entry = {"metadata": b.metadata()}
        for key, parts in fields.items():
            entry[key] = torch.cat(parts)
        out_buckets[str(b.index)] = entry
    return {"mode": mode, "step": steps.pop() if steps else 0,
            "learning_rate": float(groups[0].get("lr", 0.0)), "buckets": out_buckets}


def save_dcp(state: dict, directory: Path) -> None:
    """Write ``state`` as a single-writer DCP checkpoint (whole tensors)."""
    import torch.distributed.checkpoint as dcp

    directory.mkdir(parents=True, exist_ok=True)
    dcp.save(state, checkpoint_id=str(directory), no_dist=True)


def load_dcp(directory: Path) -> dict:
    """Read a DCP checkpoint into nested whole tensors in this process."""
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.default_planner import _EmptyStateDictLoadPlanner
    from torch.distributed.checkpoint.state_dict_loader import _load_state_dict

    state: dict = {}
    _load_state_dict(state, storage_reader=dcp.FileSystemReader(str(directory)),
                     planner=_EmptyStateDictLoadPlanner(), no_dist=True)
    return state


def load_dcp_model(directory: Path) -> dict:
    """Only the ``model`` entries of a DCP checkpoint saved as {"model": ..., ...}, read into
    CPU tensors allocated from the checkpoint's own metadata (no process group needed)."""
    import torch.distributed.checkpoint as dcp

    meta = dcp.FileSystemReader(str(directory)).read_metadata()
    target: dict = {}
    for fqn, md in meta.state_dict_metadata.items():
        if not fqn.startswith("model."):
            continue
        props = getattr(md, "properties", None)
        if props is None or not hasattr(md, "size"):
            continue
        target[fqn[len("model."):]] = torch.empty(tuple(md.size), dtype=props.dtype)
    state = {"model": target}
    dcp.load(state, checkpoint_id=str(directory), no_dist=True)
    return state["model"]
