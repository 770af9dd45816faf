"""Train the 8,192-token TinyStories BPE from the verified 500k sample, with provenance.

The output directory gets ``training.json`` (format
``nano-megatron-tokenizer-training`` v1: input path/sha256/documents, target
vocab and min frequency, resulting fingerprint). An existing output is reused
only when its provenance matches exactly. Same workflow and provenance record
as the reference (src/nano_megatron/tokenizer/tinystories.py:16-240).
"""

from __future__ import annotations

import json
import shutil
import uuid
from pathlib import Path
from typing import Any

from nano_megatron_b200.data.tinystories import (
    TINYSTORIES_SAMPLE_SEED,
    TINYSTORIES_SAMPLE_STORIES,
    TINYSTORIES_TRAIN_SHA256,
    TINYSTORIES_TRAIN_STORIES,
    validate_sample_artifact,
)

TINYSTORIES_TOKENIZER_VOCAB_SIZE = 8192
TINYSTORIES_TOKENIZER_MIN_FREQUENCY = 2
PROVENANCE_FILE = "training.json"


def _provenance(*, input_path: Path, input_sha256: str, documents: int, vocab_size: int,
                min_frequency: int, fingerprint: str) -> dict[str, Any]:
    return {"format": "nano-megatron-tokenizer-training",
            "input": {"documents": documents, "path": str(input_path.resolve()),
                      "sha256": input_sha256, "text_key": "text"},
            "tokenizer": {"fingerprint": fingerprint, "vocab_size": vocab_size},
            "training": {"min_frequency": min_frequency, "target_vocab_size": vocab_size},
            "version": 1}


def _pos(name: str, v) -> int:
    if isinstance(v, bool) or not isinstance(v, int) or v < 1:
        raise ValueError(f"{name} must be a positive integer")
    return v


def train_tinystories_tokenizer(input_path=Path("data/raw/tinystories/train_500k.jsonl"),
                                sample_metadata_path=Path(
                                    "data/raw/tinystories/train_500k.metadata.json"),
                                output_path=Path("data/tokenizers/tinystories-8k-500k"), *,
                                expected_documents: int = TINYSTORIES_SAMPLE_STORIES,
                                vocab_size: int = TINYSTORIES_TOKENIZER_VOCAB_SIZE,
                                min_frequency: int = TINYSTORIES_TOKENIZER_MIN_FREQUENCY,
                                sample_seed: int = TINYSTORIES_SAMPLE_SEED,
                                expected_source_records: int = TINYSTORIES_TRAIN_STORIES,
                                expected_source_sha256: str = TINYSTORIES_TRAIN_SHA256,
                                show_progress: bool = True) -> dict[str, Any]:
    from nano_megatron_b200.cli.tokenizer import run_train

    from .byte_bpe import ByteLevelBPETokenizer

    src, out = Path(input_path), Path(output_path)
    _pos("expected_documents", expected_documents)
    _pos("vocab_size", vocab_size)
    _pos("min_frequency", min_frequency)
    meta = validate_sample_artifact(src, Path(sample_metadata_path),
                                    sample_size=expected_documents, seed=sample_seed,
                                    expected_source_records=expected_source_records,
                                    expected_source_sha256=expected_source_sha256)
    sha = str(meta["artifact"]["sha256"])
    if out.exists():
        if not out.is_dir():
            raise FileExistsError(f"tokenizer output exists and is not a directory: {out}")
        if not (out / PROVENANCE_FILE).is_file():
            raise FileExistsError("refusing to reuse or overwrite a tokenizer without matching "
                                  f"training metadata: {out}")
        tok = ByteLevelBPETokenizer.load(out)
        want = _provenance(input_path=src, input_sha256=sha, documents=expected_documents,
                           vocab_size=vocab_size, min_frequency=min_frequency,
                           fingerprint=tok.fingerprint)
        try:
            have = json.loads((out / PROVENANCE_FILE).read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as e:
            raise ValueError(f"could not read tokenizer training metadata: {e}") from e
        if have != want:
            raise FileExistsError("existing tokenizer was trained with different corpus/"
                                  f"configuration metadata: {out}")
        if tok.vocab_size != vocab_size:
            raise ValueError(f"existing tokenizer vocabulary is not exactly {vocab_size}: "
                             f"{tok.vocab_size}")
        return {"command": "train-tinystories-tokenizer", "documents": expected_documents,
                "fingerprint": tok.fingerprint, "min_frequency": min_frequency,
                "output": str(out.resolve()), "reused": True, "vocab_size": tok.vocab_size}
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_name(f".{out.name}.tmp-{uuid.uuid4().hex}")
    try:
        r = run_train((src,), tmp, vocab_size=vocab_size, min_frequency=min_frequency,
                      text_key="text", show_progress=show_progress)
        if r["documents"] != expected_documents:
            raise RuntimeError("tokenizer trainer did not consume the required corpus size: "
                               f"{r['documents']} != {expected_documents}")
        tok = ByteLevelBPETokenizer.load(tmp)
        if tok.vocab_size != vocab_size:
            raise RuntimeError("BPE trainer did not reach the required exact vocabulary size: "
                               f"{tok.vocab_size} != {vocab_size}; use the verified 500k corpus "
                               "or lower min_frequency explicitly")
        (tmp / PROVENANCE_FILE).write_text(json.dumps(
            _provenance(input_path=src, input_sha256=sha, documents=expected_documents,
                        vocab_size=vocab_size, min_frequency=min_frequency,
                        fingerprint=tok.fingerprint),
            ensure_ascii=False, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        tmp.replace(out)
    except BaseException:
        if tmp.exists():
            shutil.rmtree(tmp)
        raise
    return {"command": "train-tinystories-tokenizer", "documents": expected_documents,
            "fingerprint": tok.fingerprint, "min_frequency": min_frequency,
            "output": str(out.resolve()), "reused": False, "vocab_size": tok.vocab_size}
