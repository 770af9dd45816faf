"""Tokenizer and corpus tools (``nano-megatron-tokenizer``): train, preprocess, split, inspect.

Subcommands and JSON reports match the reference
(src/nano_megatron/cli/tokenizer.py:21-385). ``split`` assigns each document by
the first 8 bytes of sha256("nano-megatron-jsonl-split-v1\\0<seed>\\0<text>")
against ``fraction * 2**64``, so the split is order-independent and stable.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import uuid
from collections.abc import Iterable, Iterator, Sequence
from pathlib import Path
from typing import Any

from nano_megatron_b200.data.corpus import iter_jsonl_text, preprocess_jsonl
from nano_megatron_b200.tokenizer import (
    ByteBPETrainingConfig,
    ByteLevelBPETokenizer,
    SpecialTokens,
)


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="command", required=True)
    t = sub.add_parser("train", help="learn a byte-level BPE vocabulary from JSONL documents")
    t.add_argument("--input", type=Path, action="append", required=True,
                   help="JSONL file of documents (give the flag several times for several files)")
    t.add_argument("--output", type=Path, required=True,
                   help="directory for the tokenizer artifact")
    t.add_argument("--vocab-size", type=int, default=8192,
                   help="target vocabulary size, special tokens included")
    t.add_argument("--min-frequency", type=int, default=2,
                   help="ignore merges seen fewer times than this")
    t.add_argument("--text-key", default="text", help="JSON field that holds the document text")
    d = SpecialTokens()
    t.add_argument("--unk-token", default=d.unk, help="spelling of the unknown-token marker")
    t.add_argument("--bos-token", default=d.bos, help="spelling of the begin-of-sequence marker")
    t.add_argument("--eos-token", default=d.eos, help="spelling of the end-of-sequence marker")
    t.add_argument("--pad-token", default=d.pad, help="spelling of the padding marker")
    t.add_argument("--show-progress", action="store_true", help="print trainer progress")
    pp = sub.add_parser("preprocess", help="tokenize JSONL documents into one flat token corpus")
    pp.add_argument("--input", type=Path, required=True, help="JSONL file of documents")
    pp.add_argument("--output", type=Path, required=True,
                    help="corpus file (.pt) or directory (mmap) to create")
    pp.add_argument("--tokenizer", type=Path, required=True, help="tokenizer artifact to encode with")
    pp.add_argument("--format", choices=("pt", "mmap"), default="pt",
                    help="'pt': one torch file; 'mmap': memory-mapped token array plus metadata")
    pp.add_argument("--text-key", default="text", help="JSON field that holds the document text")
    pp.add_argument("--append-eos", action=argparse.BooleanOptionalAction, default=True,
                    help="end every document with one EOS id (on by default)")
    s = sub.add_parser("split", help="divide JSONL documents into train and validation files by "
                       "a seeded hash of their text")
    s.add_argument("--input", type=Path, required=True, help="JSONL file of documents")
    s.add_argument("--train-output", type=Path, required=True, help="JSONL file for training")
    s.add_argument("--validation-output", type=Path, required=True,
                   help="JSONL file for validation")
    s.add_argument("--validation-fraction", type=float, default=0.1,
                   help="expected share of documents routed to validation")
    s.add_argument("--seed", type=int, default=1234, help="salt of the routing hash")
    s.add_argument("--text-key", default="text", help="JSON field that holds the document text")
    i = sub.add_parser("inspect", help="show how a tokenizer encodes text, or describe a mmap "
                       "corpus")
    tgt = i.add_mutually_exclusive_group(required=True)
    tgt.add_argument("--tokenizer", type=Path, help="tokenizer artifact to describe")
    tgt.add_argument("--mmap", type=Path, help="mmap corpus directory to describe")
    i.add_argument("--text", help="text to encode with --tokenizer")
    i.add_argument("--add-bos", action="store_true", help="prefix the encoding with BOS")
    i.add_argument("--add-eos", action="store_true", help="end the encoding with EOS")
    return p


class _Counted:
    def __init__(self, texts: Iterable[str]) -> None:
        self.texts, self.count = texts, 0

    def __iter__(self) -> Iterator[str]:
        for t in self.texts:
            self.count += 1
            yield t


def _inputs(paths: Sequence[Path], key: str) -> Iterator[str]:
    for p in paths:
        yield from iter_jsonl_text(p, text_key=key)


def run_train(inputs: Sequence[Path], output: Path, *, vocab_size: int = 8192,
              min_frequency: int = 2, text_key: str = "text",
              special_tokens: SpecialTokens | None = None, show_progress: bool = False
              ) -> dict[str, Any]:
    if not inputs:
        raise ValueError("tokenizer training requires at least one input JSONL path")
    ByteLevelBPETokenizer.validate_save_target(output)
    texts = _Counted(_inputs(tuple(inputs), text_key))
    tok = ByteLevelBPETokenizer.train(texts, ByteBPETrainingConfig(
        vocab_size=vocab_size, min_frequency=min_frequency,
        special_tokens=special_tokens or SpecialTokens(), show_progress=show_progress))
    if texts.count < 1:
        raise ValueError("tokenizer training corpus contains no documents")
    tok.save(output)
    return {"command": "train", "documents": texts.count, "eos_token_id": tok.eos_token_id,
            "fingerprint": tok.fingerprint, "output": str(output), "vocab_size": tok.vocab_size}


def run_preprocess(input_path: Path, output_path: Path, tokenizer_path: Path, *,
                   text_key: str = "text", append_eos: bool = True, output_format: str = "pt"
                   ) -> dict[str, Any]:
    tok = ByteLevelBPETokenizer.load(tokenizer_path)
    if output_format == "pt":
        c = preprocess_jsonl(input_path, output_path, tok, text_key=text_key,
                             append_eos=append_eos)
        return {"append_eos": c.append_eos, "command": "preprocess",
                "corpus_fingerprint": c.fingerprint, "documents": c.documents,
                "eos_token_id": c.eos_id, "output": str(output_path),
                "tokenizer_fingerprint": c.tokenizer_fingerprint,
                "tokens": int(c.tokens.numel()), "vocab_size": c.vocab_size}
    if output_format != "mmap":
        raise ValueError(f"output_format must be 'pt' or 'mmap', got {output_format!r}")
    from nano_megatron_b200.data.mmap_corpus import preprocess_jsonl_mmap

    m = preprocess_jsonl_mmap(input_path, output_path, tok, text_key=text_key,
                              append_eos=append_eos)
    return {"append_eos": m.append_eos, "command": "preprocess",
            "corpus_fingerprint": m.fingerprint, "documents": m.documents,
            "eos_token_id": m.eos_id, "format": "mmap", "output": str(output_path),
            "token_dtype": str(m.token_dtype), "tokenizer_fingerprint": m.tokenizer_fingerprint,
            "tokens": m.token_count, "vocab_size": m.vocab_size}


def split_is_validation(text: str, seed: int, fraction: float) -> bool:
    h = hashlib.sha256(f"nano-megatron-jsonl-split-v1\0{seed}\0{text}".encode()).digest()
    return int.from_bytes(h[:8], "big") < int(float(fraction) * (1 << 64))


def run_split(input_path: Path, train_output: Path, validation_output: Path, *,
              validation_fraction: float = 0.1, seed: int = 1234, text_key: str = "text"
              ) -> dict[str, Any]:
    f = validation_fraction
    if isinstance(f, bool) or not isinstance(f, (int, float)) or not 0.0 < f < 1.0:
        raise ValueError("validation_fraction must be between zero and one")
    if isinstance(seed, bool) or not isinstance(seed, int) or seed < 0:
        raise ValueError("split seed must be a non-negative integer")
    src, tr, va = input_path.resolve(), train_output.resolve(), validation_output.resolve()
    if len({src, tr, va}) != 3:
        raise ValueError("input, train output, and validation output must be distinct paths")
    for t in (tr, va):
        if t.exists():
            raise FileExistsError(f"refusing to overwrite existing split output: {t}")
        t.parent.mkdir(parents=True, exist_ok=True)
    tag = uuid.uuid4().hex
    ttmp, vtmp = tr.with_name(f".{tr.name}.{tag}.tmp"), va.with_name(f".{va.name}.{tag}.tmp")
    nt = nv = 0
    published = False
    try:
        with ttmp.open("x", encoding="utf-8", newline="\n") as tf, \
                vtmp.open("x", encoding="utf-8", newline="\n") as vf:
            for text in iter_jsonl_text(src, text_key=text_key):
                val = split_is_validation(text, seed, f)
                (vf if val else tf).write(json.dumps({text_key: text}, ensure_ascii=False,
                                                     separators=(",", ":")) + "\n")
                nv += val
                nt += not val
        if nt == 0 or nv == 0:
            raise ValueError("the deterministic split produced an empty partition; use more "
                             "documents or a different validation fraction/seed")
        ttmp.replace(tr)
        published = True
        vtmp.replace(va)
    except BaseException:
        ttmp.unlink(missing_ok=True)
        vtmp.unlink(missing_ok=True)
        if published:
            tr.unlink(missing_ok=True)
        raise
    return {"command": "split", "input": str(src), "seed": seed, "train_documents": nt,
            "train_output": str(tr), "validation_documents": nv,
            "validation_fraction": float(f), "validation_output": str(va)}


def run_inspect(tokenizer_path: Path, text: str, *, add_bos: bool = False,
                add_eos: bool = False) -> dict[str, Any]:
    tok = ByteLevelBPETokenizer.load(tokenizer_path)
    ids = tok.encode(text, add_bos=add_bos, add_eos=add_eos)
    return {"bos_token_id": tok.bos_token_id, "decoded": tok.decode(ids),
            "eos_token_id": tok.eos_token_id, "fingerprint": tok.fingerprint, "ids": ids,
            "pad_token_id": tok.pad_token_id, "tokens": [tok.id_to_token(i) for i in ids],
            "unk_token_id": tok.unk_token_id, "vocab_size": tok.vocab_size}


def run_inspect_mmap(mmap_path: Path) -> dict[str, Any]:
    from nano_megatron_b200.data.mmap_corpus import MMapTokenCorpus

    c = MMapTokenCorpus.load(mmap_path)
    return {"append_eos": c.append_eos, "corpus_fingerprint": c.fingerprint,
            "documents": c.documents, "eos_token_id": c.eos_id, "format": "mmap",
            "path": str(c.path), "token_dtype": str(c.token_dtype),
            "tokenizer_fingerprint": c.tokenizer_fingerprint, "tokens": c.token_count,
            "vocab_size": c.vocab_size}


def main(argv: Sequence[str] | None = None) -> None:
    p = parser()
    a = p.parse_args(argv)
    if a.command == "train":
        r = run_train(a.input, a.output, vocab_size=a.vocab_size, min_frequency=a.min_frequency,
                      text_key=a.text_key, special_tokens=SpecialTokens(
                          unk=a.unk_token, bos=a.bos_token, eos=a.eos_token, pad=a.pad_token),
                      show_progress=a.show_progress)
    elif a.command == "preprocess":
        r = run_preprocess(a.input, a.output, a.tokenizer, text_key=a.text_key,
                           append_eos=a.append_eos, output_format=a.format)
    elif a.command == "split":
        r = run_split(a.input, a.train_output, a.validation_output,
                      validation_fraction=a.validation_fraction, seed=a.seed,
                      text_key=a.text_key)
    else:
        if a.mmap is not None:
            if a.text is not None or a.add_bos or a.add_eos:
                p.error("inspect --mmap cannot be combined with text, BOS, or EOS options")
            r = run_inspect_mmap(a.mmap)
        else:
            if a.text is None:
                p.error("inspect --tokenizer requires --text")
            r = run_inspect(a.tokenizer, a.text, add_bos=a.add_bos, add_eos=a.add_eos)
    print(json.dumps(r, ensure_ascii=False, sort_keys=True))


if __name__ == "__main__":
    main()
