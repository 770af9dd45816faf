"""Attach the NVLink symmetric workspace that the fused SP collectives use.

Created once per TP group (a collective over that group) when training on CUDA
with TP > 1, sequence parallelism and ``kernels.fused_tp_comm``. Sizes follow
from the config: each rank's local row block is R = micro_batch * S / (CP * TP)
rows of the hidden size H; reduce-scatter staging holds TP slots of [R, H]
(two parities), the all-gather slot one [R, H] shard (two parities), the embedding
slot [R, H] rows (two parities) and the cross-entropy slots TP x (TP * R) x 3 fp32
row statistics (two parities).
"""

from __future__ import annotations

import torch


def fused_tp_rows(config, parallel) -> int:
    S = int(config.model.seq_length) // parallel.cp.size
    return int(config.training.micro_batch_size) * (S // parallel.tp.size)


def wants_fused_tp(config, parallel, device: torch.device) -> bool:
    return (device.type == "cuda" and parallel.tp.size > 1 and
            bool(config.parallel.sequence_parallel) and
            bool(getattr(config.kernels, "fused_tp_comm", True)) and
            fused_tp_rows(config, parallel) % 128 == 0 and parallel.tp.size <= 8)


def attach_tp_workspace(model: torch.nn.Module, config, parallel, device: torch.device):
    """Create the workspace (collective over TP) and set it on every GPTModel of ``model``."""
    if not wants_fused_tp(config, parallel, device):
        return None
    from nano_megatron_b200.distributed.symmetric import SymmetricWorkspace
    from nano_megatron_b200.models.gpt.model import GPTModel

    R, H = fused_tp_rows(config, parallel), int(config.model.hidden_size)
    tp = parallel.tp.size
    ws = SymmetricWorkspace.create(parallel.tp, rs_bytes=tp * R * H * 2, ag_bytes=R * H * 2,
                                   emb_bytes=R * H * 2, ce_bytes=tp * (tp * R) * 12,
                                   device=device)
    for m in model.modules():
        if isinstance(m, GPTModel):
            m.tp_workspace = ws
    return ws
