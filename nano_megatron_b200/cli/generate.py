"""Generate text on one device from an exported GPT artifact (``nano-megatron-generate``)."""

from __future__ import annotations

import argparse
import json
from collections.abc import Sequence
from pathlib import Path

from nano_megatron_b200.inference import GenerationResult, generate_from_artifact


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--model", type=Path, required=True,
                   help="artifact directory written by nano-megatron-export")
    p.add_argument("--prompt", required=True, help="text to continue")
    p.add_argument("--device", default="auto",
                   help="'auto' uses CUDA when it is available; or cpu, cuda, cuda:N")
    p.add_argument("--dtype", choices=("auto", "float32", "bfloat16", "float16"),
                   default="auto",
                   help="'auto' = fp32 on CPU, the artifact's weight dtype on CUDA")
    p.add_argument("--max-new-tokens", type=int, default=128,
                   help="stop after this many sampled tokens (or at EOS)")
    p.add_argument("--temperature", type=float, default=0.8,
                   help="softmax temperature; 0 decodes greedily")
    p.add_argument("--top-p", type=float, default=0.95,
                   help="nucleus sampling mass (1 keeps the whole distribution)")
    p.add_argument("--top-k", type=int, default=0,
                   help="sample among the k most likely tokens only (0 = no limit)")
    p.add_argument("--seed", type=int, default=1234, help="sampling RNG seed")
    p.add_argument("--add-bos", action=argparse.BooleanOptionalAction, default=True,
                   help="start the prompt with the tokenizer's BOS id (on by default)")
    p.add_argument("--kv-cache", action=argparse.BooleanOptionalAction, default=True,
                   help="reuse cached keys/values between decode steps (on by default; "
                        "--no-kv-cache recomputes the whole prefix every step)")
    p.add_argument("--json", action="store_true",
                   help="print the whole result (prompt, completion, token ids, stop reason) "
                        "as one JSON object instead of the text")
    return p


def run_generate(model: Path, prompt: str, *, device: str = "auto", dtype: str = "auto",
                 max_new_tokens: int = 128, temperature: float = 0.8, top_p: float = 0.95,
                 top_k: int = 0, seed: int = 1234, add_bos: bool = True,
                 kv_cache: bool = True) -> GenerationResult:
    return generate_from_artifact(model, prompt, device=device, dtype=dtype,
                                  max_new_tokens=max_new_tokens, temperature=temperature,
                                  top_p=top_p, top_k=top_k, seed=seed, add_bos=add_bos,
                                  use_kv_cache=kv_cache)


def main(argv: Sequence[str] | None = None) -> None:
    a = parser().parse_args(argv)
    r = run_generate(a.model, a.prompt, device=a.device, dtype=a.dtype,
                     max_new_tokens=a.max_new_tokens, temperature=a.temperature, top_p=a.top_p,
                     top_k=a.top_k, seed=a.seed, add_bos=a.add_bos, kv_cache=a.kv_cache)
    print(json.dumps(r.to_dict(), ensure_ascii=False, sort_keys=True) if a.json else r.text)


if __name__ == "__main__":
    main()
