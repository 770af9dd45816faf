"""Single-device autoregressive generation from exported GPT artifacts.

Two decoding paths over the same weights:

* ``KVCacheDecoder`` (default): the prompt is prefilled once (on CUDA through
  the tcgen05 flash-attention forward when the head size allows it), then each
  new token runs one row through every layer against a preallocated per-layer
  K/V cache ``[max_len, kv_heads, head_dim]``; QKV and gate/up projections use
  fused weight matrices, RoPE/RMSNorm use this package's kernels. Cost per
  token is O(layers * (weights + context)) instead of re-running the prefix.
* full-prefix recompute through ``GPTModel.forward`` (``use_kv_cache=False``),
  the reference's method (src/nano_megatron/inference/generation.py:151-229),
  kept as the oracle the cached path is tested against.

Sampling (greedy at temperature 0, else temperature scaling, top-k and top-p
filtering and one multinomial draw from a seeded CPU generator) follows the
reference's steps exactly (src/nano_megatron/inference/generation.py:120-148),
so a given seed picks the same tokens from the same logits.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from nano_megatron_b200.ops import functional as F

from .artifact import InferenceArtifact, load_inference_artifact, local_parallel

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@dataclass(frozen=True, slots=True)
class GenerationResult:
    prompt: str
    text: str
    completion: str
    token_ids: tuple[int, ...]
    generated_token_ids: tuple[int, ...]
    stop_reason: str

    def to_dict(self) -> dict[str, object]:
        """JSON form (the CLI's output line): every field, keys sorted, tuples as lists."""
        out = {}
        for name in sorted(self.__slots__):
            v = getattr(self, name)
            out[name] = list(v) if isinstance(v, tuple) else v
        return out


def resolve_device(value) -> torch.device:
    """``"auto"`` (CUDA when present), a device string or a ``torch.device``; only CPU and
    CUDA are accepted, and CUDA only where it exists."""
    if value == "auto":
        value = "cuda" if torch.cuda.is_available() else "cpu"
    try:
        dev = value if isinstance(value, torch.device) else torch.device(value)
    except (TypeError, RuntimeError) as e:
        raise ValueError(f"cannot parse generation device {value!r} ({e})") from e
    if dev.type not in ("cpu", "cuda"):
        raise ValueError(f"generation runs on cpu or cuda, not {dev.type}")
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError(f"device {dev} requested, but this process sees no CUDA device")
    return dev


def resolve_dtype(value: str, *, artifact: InferenceArtifact, device: torch.device):
    """``"auto"``: fp32 on CPU, the artifact's weight dtype on CUDA; else a named dtype
    (fp16 only on CUDA)."""
    if value == "auto":
        return artifact.weight_dtype if device.type == "cuda" else torch.float32
    dt = _DTYPES.get(value)
    if dt is None:
        raise ValueError(f"generation dtype {value!r}: use auto, " + ", ".join(sorted(_DTYPES)))
    if dt is torch.float16 and device.type == "cpu":
        raise ValueError("float16 generation needs CUDA; on CPU use float32 or bfloat16")
    return dt


def load_model_for_generation(artifact_path, *, device="auto", dtype: str = "auto"):
    """Artifact -> one single-device ``GPTModel`` in eval mode on ``device``."""
    from nano_megatron_b200.models.gpt.model import GPTModel

    artifact = load_inference_artifact(artifact_path)
    dev = resolve_device(device)
    model = GPTModel(artifact.model_config, parallel=local_parallel())
    model.to(dtype=resolve_dtype(dtype, artifact=artifact, device=dev))
    model.load_state_dict(artifact.state_dict, strict=True)
    model.to(device=dev).eval()
    tied = artifact.model_config.tie_embeddings
    if tied and model.lm_head.weight is not model.embedding.weight:
        raise RuntimeError("tied artifact loaded with separate embedding and LM-head tensors")
    return artifact, model, dev


def sample_next_token(logits: torch.Tensor, *, temperature: float, top_p: float, top_k: int,
                      generator: torch.Generator) -> int:
    """Next token id from one row of logits.

    Temperature 0 is greedy. Otherwise the scores are divided by the temperature, all but
    the ``top_k`` best are masked (k = 0: no cut), then the nucleus cut keeps, in
    descending order, every token whose preceding probability mass is at most ``top_p``,
    and one token is drawn from the softmax with ``generator``. These are the reference's
    steps in its order (src/nano_megatron/inference/generation.py:120-148): the same
    seed then picks the same tokens from the same logits.
    """
    z = logits.detach().to(device="cpu", dtype=torch.float32)
    if temperature == 0.0:
        return int(torch.argmax(z))
    z = z / temperature
    neg = float("-inf")
    if top_k:
        floor = z.topk(min(top_k, z.numel())).values[-1]
        z = torch.where(z < floor, torch.full_like(z, neg), z)
    if top_p < 1.0:
        ranked, order = z.sort(descending=True)
        p = ranked.softmax(-1)
        mass_before = p.cumsum(-1) - p
        ranked = ranked.masked_fill(mass_before > top_p, neg)
        z = torch.full_like(z, neg).scatter(0, order, ranked)
    probs = z.softmax(-1)
    if not bool(torch.isfinite(probs).all()) or float(probs.sum()) <= 0.0:
        raise RuntimeError("no token left to sample: the filtered distribution is empty or "
                           "not finite")
    return int(torch.multinomial(probs, 1, generator=generator))


class KVCacheDecoder:
    """Incremental decoder over a single-device ``GPTModel``'s weights."""

    def __init__(self, model, max_len: int) -> None:
        cfg = model.config
        self.model = model
        a0 = model.layers[0].attention
        self.nh, self.nkv, self.d = a0.num_heads, a0.num_kv_heads, a0.head_dim
        self.hidden = model.hidden_size
        self.eps = model.eps
        self.max_len = int(max_len)
        dev = model.embedding.weight.device
        dt = model.embedding.weight.dtype
        self.inv_freq = model.rope_inv_freq.to(dev)
        self.bias = bool(getattr(cfg, "bias", False))
        self.layers = []
        for layer in model.layers:
            at, mlp = layer.attention, layer.mlp
            wqkv = torch.cat([at.q_proj.linear.weight, at.k_proj.linear.weight,
                              at.v_proj.linear.weight]).contiguous()
            bqkv = torch.cat([at.q_proj.linear.bias, at.k_proj.linear.bias,
                              at.v_proj.linear.bias]) if self.bias else None
            wgu = torch.cat([mlp.gate_proj.linear.weight, mlp.up_proj.linear.weight]).contiguous()
            bgu = torch.cat([mlp.gate_proj.linear.bias, mlp.up_proj.linear.bias]) \
                if self.bias else None
            self.layers.append(dict(
                n1=layer.input_norm.weight, n2=layer.post_attention_norm.weight,
                wqkv=wqkv, bqkv=bqkv, wo=at.out_proj.linear.weight,
                bo=at.out_proj.linear.bias if self.bias else None, wgu=wgu, bgu=bgu,
                wd=mlp.down_proj.linear.weight,
                bd=mlp.down_proj.linear.bias if self.bias else None,
                k=torch.empty(self.max_len, self.nkv, self.d, device=dev, dtype=dt),
                v=torch.empty(self.max_len, self.nkv, self.d, device=dev, dtype=dt)))
        self.length = 0

    @staticmethod
    def _lin(x, w, b=None):
        y = x @ w.t() if not x.is_cuda else F.linear(x.contiguous(), w)
        return y + b if b is not None else y

    def _attend(self, q, kc, vc, t0: int):
        T = q.shape[0]
        if q.is_cuda and T >= 64 and self.d in (64, 128) and t0 == 0:
            o, _ = F.attention_fwd(q.unsqueeze(0), kc.unsqueeze(0), vc.unsqueeze(0),
                                   causal=True)
            return o[0].reshape(T, -1)
        rep = self.nh // self.nkv
        qf = q.float().transpose(0, 1)                                  # [nh, T, d]
        kf = kc.float().repeat_interleave(rep, 1).transpose(0, 1)       # [nh, L, d]
        vf = vc.float().repeat_interleave(rep, 1).transpose(0, 1)
        s = (qf @ kf.transpose(1, 2)) * (1.0 / math.sqrt(self.d))
        L = kc.shape[0]
        mask = torch.arange(L, device=q.device)[None, :] > \
            (torch.arange(T, device=q.device) + t0)[:, None]
        s.masked_fill_(mask, float("-inf"))
        o = torch.softmax(s, -1) @ vf
        return o.transpose(0, 1).reshape(T, -1).to(q.dtype)

    @torch.inference_mode()
    def forward(self, ids: list[int]) -> torch.Tensor:
        """Append ``ids`` to the cache; returns the logits of the last one ([V])."""
        t0, T = self.length, len(ids)
        if t0 + T > self.max_len:
            raise ValueError(f"KV cache holds {self.max_len} positions; asked for {t0 + T}")
        m = self.model
        dev = m.embedding.weight.device
        x = torch.tensor(ids, dtype=torch.long, device=dev)
        h = m.embedding.weight.index_select(0, x)
        pos = torch.arange(t0, t0 + T, dtype=torch.int32, device=dev)
        qc, kvc = self.nh * self.d, self.nkv * self.d
        for L in self.layers:
            y, _ = F.rmsnorm(h.contiguous(), L["n1"], self.eps)
            qkv = self._lin(y, L["wqkv"], L["bqkv"]).contiguous()
            F.rope_(qkv, qc + kvc, self.d, pos, self.inv_freq, inverse=False)
            L["k"][t0:t0 + T] = qkv[:, qc:qc + kvc].view(T, self.nkv, self.d)
            L["v"][t0:t0 + T] = qkv[:, qc + kvc:].view(T, self.nkv, self.d)
            q = qkv[:, :qc].view(T, self.nh, self.d)
            a = self._attend(q, L["k"][:t0 + T], L["v"][:t0 + T], t0)
            h = h + self._lin(a, L["wo"], L["bo"])
            y, _ = F.rmsnorm(h.contiguous(), L["n2"], self.eps)
            gu = self._lin(y, L["wgu"], L["bgu"])
            g, u = gu.chunk(2, dim=-1)
            h = h + self._lin((torch.nn.functional.silu(g.float()) * u.float()).to(h.dtype),
                              L["wd"], L["bd"])
        self.length = t0 + T
        y, _ = F.rmsnorm(h[-1:].contiguous(), m.final_norm.weight, self.eps)
        return self._lin(y, m.lm_head.weight)[0, :m.original_vocab_size]


def _real(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def _whole(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _check_args(prompt, max_new_tokens, temperature, top_p, top_k, seed, add_bos) -> None:
    """Argument checks of ``generate_text``: TypeError for a wrong kind, ValueError for a
    value out of range."""
    kinds = [("prompt", prompt, lambda v: isinstance(v, str), "text"),
             ("max_new_tokens", max_new_tokens, _whole, "an int"),
             ("temperature", temperature, _real, "a number"),
             ("top_p", top_p, _real, "a number"),
             ("top_k", top_k, _whole, "an int"),
             ("add_bos", add_bos, lambda v: isinstance(v, bool), "a bool")]
    for name, value, ok, want in kinds:
        if not ok(value):
            raise TypeError(f"{name} must be {want}, got {value!r}")
    ranges = [("max_new_tokens", max_new_tokens >= 1, ">= 1"),
              ("temperature", math.isfinite(float(temperature)) and temperature >= 0.0,
               "finite and >= 0"),
              ("top_p", 0.0 < float(top_p) <= 1.0, "in (0, 1]"),
              ("top_k", top_k >= 0, ">= 0")]
    for name, ok, want in ranges:
        if not ok:
            raise ValueError(f"{name} must be {want}")
    if not _whole(seed) or seed < 0:
        raise ValueError(f"seed must be an int >= 0, got {seed!r}")


def generate_text(artifact: InferenceArtifact, model, prompt: str, *, device: torch.device,
                  max_new_tokens: int = 128, temperature: float = 0.8, top_p: float = 0.95,
                  top_k: int = 0, seed: int = 1234, add_bos: bool = True,
                  use_kv_cache: bool = True) -> GenerationResult:
    _check_args(prompt, max_new_tokens, temperature, top_p, top_k, seed, add_bos)
    tok = artifact.tokenizer
    prompt_ids = tok.encode(prompt, add_bos=add_bos, add_eos=False)
    if not prompt_ids:
        raise ValueError("the prompt encodes to zero tokens: give some text or add_bos=True")
    limit = artifact.model_config.seq_length
    if len(prompt_ids) + max_new_tokens > limit:
        raise ValueError(f"{len(prompt_ids)} prompt tokens + {max_new_tokens} new tokens "
                         f"exceeds model sequence length {limit}")
    ids, new = list(prompt_ids), []
    gen = torch.Generator(device="cpu").manual_seed(seed)
    stop = "length"
    dec = KVCacheDecoder(model, len(prompt_ids) + max_new_tokens) if use_kv_cache else None
    pending = list(prompt_ids)
    with torch.inference_mode():
        for _ in range(max_new_tokens):
            if dec is not None:
                logits = dec.forward(pending)
            else:
                out = model(torch.tensor([ids], dtype=torch.long, device=device))
                logits = out.logits[0, -1, :model.original_vocab_size]
            nxt = sample_next_token(logits, temperature=float(temperature), top_p=float(top_p),
                                    top_k=top_k, generator=gen)
            ids.append(nxt)
            new.append(nxt)
            pending = [nxt]
            if nxt == tok.eos_token_id:
                stop = "eos"
                break
    return GenerationResult(prompt=prompt, text=tok.decode(ids, skip_special_tokens=True),
                            completion=tok.decode(new, skip_special_tokens=True),
                            token_ids=tuple(ids), generated_token_ids=tuple(new),
                            stop_reason=stop)


def generate_from_artifact(artifact_path, prompt: str, *, device="auto", dtype: str = "auto",
                           max_new_tokens: int = 128, temperature: float = 0.8,
                           top_p: float = 0.95, top_k: int = 0, seed: int = 1234,
                           add_bos: bool = True, use_kv_cache: bool = True) -> GenerationResult:
    artifact, model, dev = load_model_for_generation(artifact_path, device=device, dtype=dtype)
    return generate_text(artifact, model, prompt, device=dev, max_new_tokens=max_new_tokens,
                         temperature=temperature, top_p=top_p, top_k=top_k, seed=seed,
                         add_bos=add_bos, use_kv_cache=use_kv_cache)
