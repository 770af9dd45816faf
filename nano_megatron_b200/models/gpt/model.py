"""Decoder-only GPT: modules (parameter layout identical to the reference) and
the fused training forward.

Module tree and state-dict keys match the reference's GPTModel
(src/nano_megatron/models/gpt/model.py:40-250, layer.py, attention.py, mlp.py):
``embedding.weight``, ``layers.{i}.input_norm.weight``,
``layers.{i}.attention.{q,k,v}_proj.linear.weight``,
``layers.{i}.attention.out_proj.linear.weight`` (+``out_proj.bias``),
``layers.{i}.post_attention_norm.weight``,
``layers.{i}.mlp.{gate,up}_proj.linear.weight``, ``layers.{i}.mlp.down_proj.linear.weight``,
``final_norm.weight``, ``lm_head.weight`` (the embedding Parameter when tied).
Parameters are created in the same order with the same initialisers, so the
same seed gives the same initial weights.

Execution differs: each layer runs as two fused autograd functions
(:mod:`.blocks`) over sequence-major activations.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn

from nano_megatron_b200.nn.activation_checkpoint import activation_checkpoint
from nano_megatron_b200.nn.dropout import make_dropout
from nano_megatron_b200.nn.norms import RMSNorm
from nano_megatron_b200.nn.rotary import rope_inv_freq
from nano_megatron_b200.utils.profiling import nvtx_range
from nano_megatron_b200.tensor_parallel.embedding import VocabParallelEmbedding
from nano_megatron_b200.tensor_parallel.layers import (
    ColumnParallelLinear,
    RowParallelLinear,
    VocabParallelLinear,
)

from . import blocks as B


def _cfg(config, *names, default=None):
    for n in names:
        if hasattr(config, n):
            return getattr(config, n)
        if isinstance(config, dict) and n in config:
            return config[n]
    return default


@dataclass
class GPTOutput:
    """``logits`` stay vocabulary-sharded ([B, S, V/TP]) when present."""

    logits: torch.Tensor | None
    loss: torch.Tensor | None
    hidden_states: torch.Tensor


class GPTAttention(nn.Module):
    def __init__(self, config, layer_index: int, *, parallel, sequence_parallel: bool) -> None:
        super().__init__()
        self.layer_index = layer_index
        self.hidden_size = int(_cfg(config, "hidden_size"))
        self.num_heads = int(_cfg(config, "heads", "num_attention_heads"))
        kv = _cfg(config, "num_kv_heads", "kv_heads")
        self.num_kv_heads = int(kv if kv is not None else self.num_heads)
        tp = parallel.tp.size
        if self.hidden_size % self.num_heads or self.num_heads % self.num_kv_heads:
            raise ValueError("invalid head configuration")
        if self.num_heads % tp or self.num_kv_heads % tp:
            raise ValueError("query and KV head counts must both be divisible by TP size")
        self.head_dim = self.hidden_size // self.num_heads
        self.local_num_heads = self.num_heads // tp
        self.local_num_kv_heads = self.num_kv_heads // tp
        bias = bool(_cfg(config, "bias", "linear_bias", default=False))
        kvh = self.num_kv_heads * self.head_dim
        common = dict(parallel=parallel, bias=bias, sequence_parallel=False,
                      disable_input_gradient_reduce=sequence_parallel)
        self.q_proj = ColumnParallelLinear(self.hidden_size, self.hidden_size, **common)
        self.k_proj = ColumnParallelLinear(self.hidden_size, kvh, **common)
        self.v_proj = ColumnParallelLinear(self.hidden_size, kvh, **common)
        self.out_proj = RowParallelLinear(self.hidden_size, self.hidden_size, parallel=parallel,
                                          bias=bias, input_is_parallel=True,
                                          sequence_parallel=sequence_parallel)
        self.rope_theta = float(_cfg(config, "rope_theta", default=10_000.0))


class GPTMLP(nn.Module):
    def __init__(self, config, layer_index: int, *, parallel, sequence_parallel: bool) -> None:
        super().__init__()
        hidden = int(_cfg(config, "hidden_size"))
        ffn = int(_cfg(config, "ffn_hidden_size"))
        bias = bool(_cfg(config, "bias", "linear_bias", default=False))
        common = dict(parallel=parallel, bias=bias, sequence_parallel=False,
                      disable_input_gradient_reduce=sequence_parallel)
        self.gate_proj = ColumnParallelLinear(hidden, ffn, **common)
        self.up_proj = ColumnParallelLinear(hidden, ffn, **common)
        self.down_proj = RowParallelLinear(ffn, hidden, parallel=parallel, bias=bias,
                                           input_is_parallel=True,
                                           sequence_parallel=sequence_parallel)
        self.ffn_local = ffn // parallel.tp.size


class GPTLayer(nn.Module):
    """Pre-norm block: h += attn(norm1(h)); h += mlp(norm2(h))."""

    def __init__(self, config, layer_index: int, *, parallel, sequence_parallel: bool,
                 rng=None, checkpoint_config=None, components=None) -> None:
        super().__init__()
        self.layer_index = layer_index
        self.rng = rng
        self.checkpoint_config = checkpoint_config
        eps = float(_cfg(config, "norm_epsilon", default=1e-5))
        hidden = int(_cfg(config, "hidden_size"))
        build_norm = getattr(components, "build_norm", None)
        self.input_norm = build_norm(config) if build_norm else RMSNorm(hidden, eps)
        self.attention = GPTAttention(config, layer_index, parallel=parallel,
                                      sequence_parallel=sequence_parallel)
        self.post_attention_norm = build_norm(config) if build_norm else RMSNorm(hidden, eps)
        build_mlp = getattr(components, "build_mlp", None)
        self.mlp = build_mlp(config, layer_index, parallel=parallel,
                             sequence_parallel=sequence_parallel) if build_mlp else \
            GPTMLP(config, layer_index, parallel=parallel, sequence_parallel=sequence_parallel)
        self.dropout = float(_cfg(config, "dropout", "hidden_dropout", default=0.0))
        if sequence_parallel:
            self.input_norm.weight.sequence_parallel_grad = True
            self.post_attention_norm.weight.sequence_parallel_grad = True

    def _selective(self, name: str) -> bool:
        c = self.checkpoint_config
        return (c is not None and str(getattr(c, "mode", "none")) == "selective"
                and name in tuple(getattr(c, "selective_ops", ())) and self.training)

    def forward(self, h, *, attn_spec, mlp_spec, mb, inv_freq, token_offset: int = 0):
        a = self.attention
        drop_a = make_dropout(self.dropout, training=self.training, rng=self.rng,
                              layer=self.layer_index, microbatch=mb.microbatch_index,
                              global_token_offset=token_offset, op="attention_residual")
        drop_m = make_dropout(self.dropout, training=self.training, rng=self.rng,
                              layer=self.layer_index, microbatch=mb.microbatch_index,
                              global_token_offset=token_offset, op="mlp_residual")

        m = self.mlp
        b_qkv = (a.q_proj.bias, a.k_proj.bias, a.v_proj.bias) \
            if a.q_proj.bias is not None else None
        b_gu = (m.gate_proj.bias, m.up_proj.bias) if m.gate_proj.bias is not None else None

        def attn(x):
            mb.extra["layer"] = self.layer_index    # context parallelism keys its K/V slot
            return B.AttentionBlockFn.apply(
                x, self.input_norm.weight, a.q_proj.weight, a.k_proj.weight, a.v_proj.weight,
                a.out_proj.weight, a.out_proj.bias, attn_spec, mb, inv_freq, drop_a, b_qkv)

        def mlp(x):
            return B.MLPBlockFn.apply(x, self.post_attention_norm.weight, m.gate_proj.weight,
                                      m.up_proj.weight, m.down_proj.weight, m.down_proj.bias,
                                      mlp_spec, drop_m, b_gu)

        off = bool(getattr(self.checkpoint_config, "offload_saved_tensors", False))
        h = activation_checkpoint(attn, h, offload_saved_tensors=off) \
            if self._selective("attention") else attn(h)
        h = activation_checkpoint(mlp, h, offload_saved_tensors=off) \
            if self._selective("mlp") else mlp(h)
        return h


class GPTModel(nn.Module):
    def __init__(self, config, *, parallel, kernels=None, rng=None, components=None,
                 cp_attention=None, parameter_domains=None, activation_checkpoint_config=None,
                 sequence_parallel: bool | None = None, layer_start: int = 0,
                 layer_end: int | None = None, owns_embedding: bool = True,
                 owns_final_norm: bool = True, owns_lm_head: bool = True) -> None:
        super().__init__()
        self.config = config
        self.parallel = parallel
        self.rng = rng
        self.activation_checkpoint_config = activation_checkpoint_config
        sp = bool(getattr(parallel, "sequence_parallel", False)) if sequence_parallel is None \
            else bool(sequence_parallel)
        self.sequence_parallel = sp and parallel.tp.size > 1
        self.hidden_size = int(_cfg(config, "hidden_size"))
        self.num_layers = int(_cfg(config, "layers", "num_layers"))
        self.original_vocab_size = int(_cfg(config, "vocab_size"))
        tp = parallel.tp.size
        self.padded_vocab_size = math.ceil(self.original_vocab_size / tp) * tp
        self.dropout = float(_cfg(config, "dropout", "embedding_dropout", default=0.0))
        self.eps = float(_cfg(config, "norm_epsilon", default=1e-5))
        self.owns_embedding, self.owns_final_norm, self.owns_lm_head = \
            owns_embedding, owns_final_norm, owns_lm_head
        self.layer_start = layer_start
        self.layer_end = self.num_layers if layer_end is None else layer_end
        if not 0 <= self.layer_start < self.layer_end <= self.num_layers:
            raise ValueError(f"invalid layer range [{self.layer_start}, {self.layer_end}) for "
                             f"{self.num_layers} layers")
        init_std = float(_cfg(config, "init_std", default=0.02))
        self.embedding = VocabParallelEmbedding(
            self.padded_vocab_size, self.hidden_size, parallel=parallel,
            sequence_parallel=self.sequence_parallel, init_std=init_std) if owns_embedding else None
        self.layers = nn.ModuleList([
            GPTLayer(config, i, parallel=parallel, sequence_parallel=self.sequence_parallel,
                     rng=rng, checkpoint_config=activation_checkpoint_config,
                     components=components)
            for i in range(self.layer_start, self.layer_end)])
        self.final_norm = RMSNorm(self.hidden_size, self.eps) if owns_final_norm else None
        if self.final_norm is not None and self.sequence_parallel:
            self.final_norm.weight.sequence_parallel_grad = True
        tied = self.embedding.weight if (bool(_cfg(config, "tie_embeddings", default=True))
                                         and self.embedding is not None) else None
        self.lm_head = VocabParallelLinear(
            self.hidden_size, self.padded_vocab_size, parallel=parallel,
            sequence_parallel=self.sequence_parallel, weight=tied,
            init_std=init_std) if owns_lm_head else None
        self.cp_attention = cp_attention
        a0 = self.layers[0].attention
        self.head_dim = a0.head_dim
        self.register_buffer("rope_inv_freq", rope_inv_freq(a0.head_dim, a0.rope_theta),
                             persistent=False)
        self._pos_cache: dict = {}

    # ------------------------------------------------------------------ helpers
    def _tp_info(self) -> B.TPInfo:
        tp = self.parallel.tp
        return B.TPInfo(tp if tp.size > 1 else None, tp.size, self.sequence_parallel,
                        getattr(self, "tp_workspace", None))

    def _specs(self):
        tpi = self._tp_info()
        a0 = self.layers[0].attention
        core = self.cp_attention if self.cp_attention is not None else B.LocalAttentionCore()
        attn = B.AttnSpec(self.hidden_size, a0.local_num_heads, a0.local_num_kv_heads,
                          a0.head_dim, self.eps, tpi, core)
        mlp = B.MLPSpec(self.hidden_size, self.layers[0].mlp.ffn_local, self.eps, tpi)
        return tpi, attn, mlp

    def _positions(self, seq: int, device, position_ids) -> torch.Tensor:
        if position_ids is not None:
            pos = position_ids.reshape(-1, position_ids.shape[-1])[0]
            return pos.to(device=device, dtype=torch.int32).contiguous()
        cp = self.parallel.cp
        key = (seq, device, cp.rank, cp.size,
               getattr(self.cp_attention, "load_balance", False))
        pos = self._pos_cache.get(key)
        if pos is None:
            if self.cp_attention is not None and hasattr(self.cp_attention, "local_positions"):
                pos = self.cp_attention.local_positions(seq, cp.rank, cp.size)
            else:
                pos = torch.arange(cp.rank * seq, cp.rank * seq + seq)
            pos = pos.to(device=device, dtype=torch.int32)
            self._pos_cache[key] = pos
        return pos

    def _checkpoint_layer(self, layer) -> bool:
        c = self.activation_checkpoint_config
        if c is None or str(getattr(c, "mode", "none")) != "full" or not self.training:
            return False
        return layer.layer_index % int(getattr(c, "block_interval", 1)) == 0

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: torch.Tensor | None = None, *, labels: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None,
                hidden_states: torch.Tensor | None = None,
                microbatch_index: int = 0) -> GPTOutput:
        """``input_ids``/``labels`` are ``[B, S_local]``; ``hidden_states`` (between
        pipeline stages) are sequence-major ``[S_local(/TP under SP), B, H]``."""
        tpi, attn_spec, mlp_spec = self._specs()
        if self.embedding is not None:
            if input_ids is None:
                raise ValueError("the first pipeline stage requires input_ids")
            Bsz, S = input_ids.shape
            device = self.embedding.weight.device
            ids = input_ids.t().reshape(-1).to(device=device, dtype=torch.long)
            h = B.EmbeddingFn.apply(ids, self.embedding.weight, self.embedding.vocab_start_index,
                                    tpi)
            h = h.view(-1, Bsz, self.hidden_size)
            if self.dropout > 0 and self.training:
                from nano_megatron_b200.nn.dropout import parallel_dropout

                h = parallel_dropout(h, self.dropout, training=True, rng=self.rng, layer=0,
                                     microbatch=microbatch_index, op="embedding")
        else:
            if hidden_states is None:
                raise ValueError("a non-first pipeline stage requires hidden_states")
            h = hidden_states
            Bsz = h.shape[1]
            S = h.shape[0] * (tpi.size if self.sequence_parallel else 1)
            device = h.device
        mb = B.MicrobatchInfo(batch=Bsz, seq=S, positions=self._positions(S, device, position_ids),
                              microbatch_index=microbatch_index)
        inv_freq = self.rope_inv_freq
        if inv_freq.device != device:
            self.rope_inv_freq = inv_freq = inv_freq.to(device)
        for layer in self.layers:
            with nvtx_range(f"layer {layer.layer_index}"):
                if self._checkpoint_layer(layer):
                    h = activation_checkpoint(
                        lambda x, lyr=layer: lyr(x, attn_spec=attn_spec, mlp_spec=mlp_spec,
                                                 mb=mb, inv_freq=inv_freq),
                        h, offload_saved_tensors=bool(getattr(
                            self.activation_checkpoint_config, "offload_saved_tensors", False)))
                else:
                    h = layer(h, attn_spec=attn_spec, mlp_spec=mlp_spec, mb=mb,
                              inv_freq=inv_freq)
        if self.lm_head is None:
            return GPTOutput(logits=None, loss=None, hidden_states=h)
        if labels is not None:
            lab = labels.t().reshape(-1).to(device=device, dtype=torch.long)
            if self.final_norm is None:
                raise ValueError("the LM-head stage must own the final norm")
            loss = B.HeadLossFn.apply(h, self.final_norm.weight, self.lm_head.weight, lab,
                                      self.eps, tpi)
            return GPTOutput(logits=None, loss=loss, hidden_states=h)
        logits = self.compute_logits(h)
        return GPTOutput(logits=logits, loss=None, hidden_states=h)

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        """Vocab-sharded logits ``[B, S, V/TP]`` (no gradient path)."""
        with torch.no_grad():
            from nano_megatron_b200.ops import functional as F

            tpi = self._tp_info()
            Bsz = h.shape[1]
            h2 = h.reshape(-1, self.hidden_size)
            if self.final_norm is not None:
                h2, _ = F.rmsnorm(h2.contiguous(), self.final_norm.weight, self.eps)
            hg = tpi.gather(h2)
            logits = F.linear(hg, self.lm_head.weight)
            return logits.view(-1, Bsz, logits.shape[-1]).transpose(0, 1)
