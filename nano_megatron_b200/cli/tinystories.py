"""TinyStories preparation (``nano-megatron-tinystories``): download, train-tokenizer, prepare-corpus.

One entry point for the three reference helper scripts
(scripts/download_tinystories.py, scripts/train_tinystories_tokenizer.py,
scripts/prepare_tinystories_corpus.py); each subcommand prints one JSON report.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from collections.abc import Sequence
from pathlib import Path


class _Progress:
    def __init__(self) -> None:
        self._last = -1

    def __call__(self, done: int, total: int) -> None:
        pct = int(100 * done / max(total, 1))
        if pct != self._last:
            self._last = pct
            print(f"\r{done}/{total} ({pct}%)", end="", file=sys.stderr, flush=True)


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="command", required=True)
    d = sub.add_parser("download", help="download the pinned train source and publish the "
                       "exact 500k JSONL sample")
    d.add_argument("--data-dir", type=Path, default=Path("data/raw/tinystories"))
    d.add_argument("--url", action="append", default=None, help="mirror URL (repeatable)")
    d.add_argument("--quiet", action="store_true")
    t = sub.add_parser("train-tokenizer", help="train the 8k BPE from the verified sample")
    t.add_argument("--input", type=Path, default=Path("data/raw/tinystories/train_500k.jsonl"))
    t.add_argument("--sample-metadata", type=Path,
                   default=Path("data/raw/tinystories/train_500k.metadata.json"))
    t.add_argument("--output", type=Path, default=Path("data/tokenizers/tinystories-8k-500k"))
    t.add_argument("--threads", type=int, default=min(16, os.cpu_count() or 1))
    t.add_argument("--quiet", action="store_true")
    c = sub.add_parser("prepare-corpus", help="download train/validation and build the full "
                       "mmap corpora")
    c.add_argument("--data-dir", type=Path, default=Path("data/raw/tinystories"))
    c.add_argument("--tokenizer", type=Path, default=Path("data/tokenizers/tinystories-8k-500k"))
    c.add_argument("--output", type=Path, default=Path("data/processed/tinystories-full-8k"))
    c.add_argument("--train-url", action="append", default=None)
    c.add_argument("--validation-url", action="append", default=None)
    c.add_argument("--quiet", action="store_true")
    return p


def main(argv: Sequence[str] | None = None) -> None:
    a = parser().parse_args(argv)
    prog = None if a.quiet else _Progress()
    if a.command == "download":
        from nano_megatron_b200.data.tinystories import (TINYSTORIES_TRAIN_URLS,
                                                          prepare_tinystories_500k)

        r = prepare_tinystories_500k(a.data_dir, urls=a.url or TINYSTORIES_TRAIN_URLS,
                                     progress=prog)
    elif a.command == "train-tokenizer":
        if a.threads < 1:
            raise ValueError("--threads must be positive")
        os.environ.setdefault("RAYON_NUM_THREADS", str(a.threads))
        from nano_megatron_b200.tokenizer.tinystories import train_tinystories_tokenizer

        r = train_tinystories_tokenizer(a.input, a.sample_metadata, a.output,
                                        show_progress=not a.quiet)
    else:
        from nano_megatron_b200.data.tinystories import (TINYSTORIES_TRAIN_URLS,
                                                          TINYSTORIES_VALIDATION_URLS)
        from nano_megatron_b200.data.tinystories_corpus import prepare_tinystories_corpus

        r = prepare_tinystories_corpus(a.data_dir, a.tokenizer, a.output,
                                       train_urls=a.train_url or TINYSTORIES_TRAIN_URLS,
                                       validation_urls=a.validation_url or
                                       TINYSTORIES_VALIDATION_URLS, progress=prog)
    if prog is not None:
        print(file=sys.stderr)
    print(json.dumps(r, ensure_ascii=False, sort_keys=True))


if __name__ == "__main__":
    main()
