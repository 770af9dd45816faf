"""ZeRO-3: parameters, gradients and optimizer state sharded over the replica group.

Each transformer layer (and the embedding / head) is its own bucket. A layer's
bf16 parameters are all-gathered from the owners' shards right before its
forward (the next layer's gather is prefetched on a side stream) and released
after it when ``reshard_after_forward``; they are gathered again before its
backward, and its fp32 gradients are reduce-scattered to the owners, which run
the sharded AdamW on fp32 masters. The reference wraps the stage in one FSDP2
unit instead (src/nano_megatron/data_parallel/zero3.py:152-165).
"""

from __future__ import annotations

from .strategies import Zero2Strategy


class Zero3Strategy(Zero2Strategy):
    mode = "zero3"
    graph_safe_microbatches = False
    reduce_scatter = True
