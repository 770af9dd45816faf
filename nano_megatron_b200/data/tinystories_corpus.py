"""Full TinyStories train/validation mmap corpora as one validated, atomically published directory.

Layout: ``train.mmap/`` and ``validation.mmap/`` (mmap corpora, EOS appended),
``manifest.json`` (artifact ``nano_megatron.tinystories_corpus`` v1: source
revisions, the verified source files, the tokenizer identity, each corpus's
metadata) and ``.complete``. A rebuild into an existing directory validates
and reuses it when it was built from the same sources, else refuses. Same
layout and manifest as the reference
(src/nano_megatron/data/tinystories_corpus.py:36-488).
"""

from __future__ import annotations

import json
import os
import shutil
import tempfile
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any

from nano_megatron_b200.tokenizer import ByteLevelBPETokenizer

from .mmap_corpus import MMapTokenCorpus, preprocess_texts_mmap
from .tinystories import (
    TINYSTORIES_CANONICAL_REVISION,
    TINYSTORIES_DELIMITER,
    TINYSTORIES_MIRROR_REVISION,
    TINYSTORIES_TRAIN_BYTES,
    TINYSTORIES_TRAIN_SHA256,
    TINYSTORIES_TRAIN_STORIES,
    TINYSTORIES_TRAIN_URLS,
    TINYSTORIES_VALIDATION_BYTES,
    TINYSTORIES_VALIDATION_SHA256,
    TINYSTORIES_VALIDATION_STORIES,
    TINYSTORIES_VALIDATION_URLS,
    FileVerification,
    ProgressCallback,
    download_pinned_file,
    iter_delimited_stories,
    verify_file,
)

ARTIFACT_NAME = "nano_megatron.tinystories_corpus"
ARTIFACT_VERSION = 1
COMPLETE = ".complete"
MANIFEST = "manifest.json"
TRAIN_DIR = "train.mmap"
VALIDATION_DIR = "validation.mmap"
EXPECTED_VOCAB = 8192
_TOP_KEYS = {"artifact", "corpora", "format_version", "source_revision", "sources", "tokenizer"}


class TinyStoriesCorpusError(ValueError):
    """A full TinyStories artifact violates its contract."""


def _obj(v: Any, what: str) -> Mapping:
    if not isinstance(v, Mapping):
        raise TinyStoriesCorpusError(f"{what} must be an object")
    return v


def _text(v: Any, what: str) -> str:
    if not isinstance(v, str) or not v:
        raise TinyStoriesCorpusError(f"{what} must be a non-empty string")
    return v


def _subdir(root: Path, v: Any, what: str) -> Path:
    rel = Path(_text(v, what))
    if rel.is_absolute() or ".." in rel.parts:
        raise TinyStoriesCorpusError(f"{what} must be a safe relative path")
    if not (root / rel).is_dir():
        raise TinyStoriesCorpusError(f"{what} does not exist: {root / rel}")
    return root / rel


def _corpus_entry(directory: str, c: MMapTokenCorpus) -> dict[str, Any]:
    return {"append_eos": c.append_eos, "directory": directory,
            "document_offsets_sha256": c.document_offsets_sha256, "documents": c.documents,
            "fingerprint": c.fingerprint, "token_count": c.token_count,
            "token_dtype": c.token_dtype.str, "tokens_sha256": c.tokens_sha256}


def _source_entry(v: FileVerification, stories: int) -> dict[str, Any]:
    return {"path": str(v.path), "sha256": v.sha256, "size_bytes": v.size_bytes,
            "stories": stories, "story_delimiter": TINYSTORIES_DELIMITER.decode("ascii")}


def _load(path: Path, what: str) -> MMapTokenCorpus:
    try:
        return MMapTokenCorpus.load(path)
    except (OSError, ValueError) as e:
        raise TinyStoriesCorpusError(f"could not validate {what}: {e}") from e


def validate_tinystories_corpus(path, *, tokenizer_path=None) -> dict[str, Any]:
    d = Path(path).resolve()
    if not d.is_dir() or not (d / COMPLETE).is_file():
        raise TinyStoriesCorpusError(f"TinyStories corpus is incomplete or missing: {d}")
    have, want = {e.name for e in d.iterdir()}, {COMPLETE, MANIFEST, TRAIN_DIR, VALIDATION_DIR}
    if have != want:
        raise TinyStoriesCorpusError(f"TinyStories corpus directory entries differ: {have} != "
                                     f"{want}")
    try:
        m = json.loads((d / MANIFEST).read_text(encoding="utf-8"))
    except (OSError, UnicodeDecodeError, json.JSONDecodeError) as e:
        raise TinyStoriesCorpusError(f"could not read TinyStories corpus manifest: {e}") from e
    if not isinstance(m, dict) or set(m) != _TOP_KEYS:
        raise TinyStoriesCorpusError("TinyStories corpus manifest has invalid top-level keys")
    if m.get("artifact") != ARTIFACT_NAME:
        raise TinyStoriesCorpusError("TinyStories corpus artifact name is unsupported")
    if m.get("format_version") != ARTIFACT_VERSION:
        raise TinyStoriesCorpusError("TinyStories corpus format version is unsupported")
    if m.get("source_revision") != {"canonical": TINYSTORIES_CANONICAL_REVISION,
                                    "mirror": TINYSTORIES_MIRROR_REVISION}:
        raise TinyStoriesCorpusError("TinyStories corpus source revision is invalid")
    tok = _obj(m.get("tokenizer"), "tokenizer")
    if set(tok) != {"eos_token_id", "fingerprint", "path", "vocab_size"}:
        raise TinyStoriesCorpusError("tokenizer manifest fields are invalid")
    fp = _text(tok.get("fingerprint"), "tokenizer.fingerprint")
    _text(tok.get("path"), "tokenizer.path")
    vocab, eos = tok.get("vocab_size"), tok.get("eos_token_id")
    if isinstance(vocab, bool) or not isinstance(vocab, int) or vocab < 1:
        raise TinyStoriesCorpusError("tokenizer.vocab_size must be a positive integer")
    if isinstance(eos, bool) or not isinstance(eos, int) or not 0 <= eos < vocab:
        raise TinyStoriesCorpusError("tokenizer.eos_token_id is invalid")
    if tokenizer_path is not None:
        t = ByteLevelBPETokenizer.load(tokenizer_path)
        if (t.fingerprint, t.vocab_size, t.eos_token_id) != (fp, vocab, eos):
            raise TinyStoriesCorpusError("TinyStories corpus tokenizer does not match the "
                                         "requested tokenizer artifact")
    corpora = _obj(m.get("corpora"), "corpora")
    if set(corpora) != {"train", "validation"}:
        raise TinyStoriesCorpusError("corpora must contain train and validation")
    loaded = {}
    for name in ("train", "validation"):
        e = _obj(corpora[name], f"corpora.{name}")
        loaded[name] = (e, _load(_subdir(d, e.get("directory"), f"corpora.{name}.directory"),
                                 f"{name} mmap"))
    try:
        for name, (e, c) in loaded.items():
            if dict(e) != _corpus_entry(str(e.get("directory")), c):
                raise TinyStoriesCorpusError(f"corpora.{name} metadata does not match its mmap "
                                             "artifact")
            if not c.append_eos:
                raise TinyStoriesCorpusError(f"{name} mmap must append EOS")
            if c.tokenizer_fingerprint != fp:
                raise TinyStoriesCorpusError(f"{name} tokenizer fingerprint does not match")
            if c.vocab_size != vocab or c.eos_id != eos:
                raise TinyStoriesCorpusError(f"{name} tokenizer metadata does not match")
        if loaded["train"][1].fingerprint == loaded["validation"][1].fingerprint:
            raise TinyStoriesCorpusError("train and validation mmap fingerprints must differ")
    finally:
        for _, c in loaded.values():
            c.close()
    sources = _obj(m.get("sources"), "sources")
    if set(sources) != {"train", "validation"}:
        raise TinyStoriesCorpusError("sources must contain train and validation")
    for name in ("train", "validation"):
        s = _obj(sources[name], f"sources.{name}")
        if set(s) != {"path", "sha256", "size_bytes", "stories", "story_delimiter"}:
            raise TinyStoriesCorpusError(f"sources.{name} fields are invalid")
        _text(s.get("path"), f"sources.{name}.path")
        dg = _text(s.get("sha256"), f"sources.{name}.sha256")
        try:
            ok = len(dg) == 64 and bytes.fromhex(dg) is not None
        except ValueError:
            ok = False
        if not ok:
            raise TinyStoriesCorpusError(f"sources.{name}.sha256 must be a SHA256 digest")
        for k in ("size_bytes", "stories"):
            v = s.get(k)
            if isinstance(v, bool) or not isinstance(v, int) or v < 1:
                raise TinyStoriesCorpusError(f"sources.{name}.{k} must be a positive integer")
        if s.get("story_delimiter") != TINYSTORIES_DELIMITER.decode("ascii"):
            raise TinyStoriesCorpusError(f"sources.{name}.story_delimiter is invalid")
    if sources["train"].get("sha256") == sources["validation"].get("sha256"):
        raise TinyStoriesCorpusError("train and validation source SHA256 must differ")
    return m


def _target(d: Path) -> bool:
    if d.is_symlink():
        raise FileExistsError(f"refusing to replace TinyStories corpus symlink: {d}")
    if not d.exists():
        return False
    if not d.is_dir():
        raise FileExistsError(f"TinyStories corpus output already exists: {d}")
    return not any(d.iterdir())


def build_tinystories_corpus(train_source, validation_source, tokenizer_path, output_path, *,
                             train_verification: FileVerification,
                             validation_verification: FileVerification,
                             expected_train_stories: int, expected_validation_stories: int,
                             expected_vocab_size: int = EXPECTED_VOCAB) -> dict[str, Any]:
    tr, va = Path(train_source).resolve(), Path(validation_source).resolve()
    if tr == va:
        raise ValueError("train and validation sources must be distinct")
    checked = []
    for p, v in ((tr, train_verification), (va, validation_verification)):
        if v.path.resolve() != p:
            raise ValueError("source verification describes a different path")
        checked.append(verify_file(p, expected_size=v.size_bytes, expected_sha256=v.sha256))
    trv, vav = checked
    if trv.sha256 == vav.sha256:
        raise ValueError("train and validation source SHA256 must differ")
    tok_src = Path(tokenizer_path).resolve()
    tok = ByteLevelBPETokenizer.load(tok_src)
    if tok.vocab_size != expected_vocab_size:
        raise ValueError(f"TinyStories tokenizer vocab size {tok.vocab_size} != "
                         f"{expected_vocab_size}")
    dest = Path(output_path).resolve()
    was_empty = _target(dest)
    if dest.exists() and not was_empty:
        m = validate_tinystories_corpus(dest, tokenizer_path=tok_src)
        if (m["sources"]["train"] != _source_entry(trv, expected_train_stories) or
                m["sources"]["validation"] != _source_entry(vav, expected_validation_stories) or
                m["corpora"]["train"].get("documents") != expected_train_stories or
                m["corpora"]["validation"].get("documents") != expected_validation_stories):
            raise FileExistsError("existing TinyStories corpus was built from different sources "
                                  "or counts")
        return {"command": "prepare-tinystories-corpus", "manifest": m, "output": str(dest),
                "reused": True}
    dest.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=f".{dest.name}.tmp-", dir=dest.parent))
    removed = False
    try:
        t = preprocess_texts_mmap(iter_delimited_stories(tr), tmp / TRAIN_DIR, tok)
        v = preprocess_texts_mmap(iter_delimited_stories(va), tmp / VALIDATION_DIR, tok)
        for name, c, want in (("train", t, expected_train_stories),
                              ("validation", v, expected_validation_stories)):
            if c.documents != want:
                raise TinyStoriesCorpusError(f"{name} source emitted {c.documents} stories, "
                                             f"expected {want}")
        m = {"artifact": ARTIFACT_NAME,
             "corpora": {"train": _corpus_entry(TRAIN_DIR, t),
                         "validation": _corpus_entry(VALIDATION_DIR, v)},
             "format_version": ARTIFACT_VERSION,
             "source_revision": {"canonical": TINYSTORIES_CANONICAL_REVISION,
                                 "mirror": TINYSTORIES_MIRROR_REVISION},
             "sources": {"train": _source_entry(trv, t.documents),
                         "validation": _source_entry(vav, v.documents)},
             "tokenizer": {"eos_token_id": tok.eos_token_id, "fingerprint": tok.fingerprint,
                           "path": str(tok_src), "vocab_size": tok.vocab_size}}
        (tmp / MANIFEST).write_text(json.dumps(m, ensure_ascii=False, indent=2, sort_keys=True)
                                    + "\n", encoding="utf-8")
        (tmp / COMPLETE).write_text("complete\n", encoding="utf-8")
        validate_tinystories_corpus(tmp, tokenizer_path=tok_src)
        if was_empty:
            dest.rmdir()
            removed = True
        elif dest.exists() or dest.is_symlink():
            raise FileExistsError(f"TinyStories corpus output already exists: {dest}")
        os.replace(tmp, dest)
    except BaseException:
        if removed and not dest.exists():
            dest.mkdir()
        raise
    finally:
        if tmp.exists():
            shutil.rmtree(tmp)
    return {"command": "prepare-tinystories-corpus",
            "manifest": validate_tinystories_corpus(dest, tokenizer_path=tok_src),
            "output": str(dest), "reused": False}


def prepare_tinystories_corpus(data_dir=Path("data/raw/tinystories"),
                               tokenizer_path=Path("data/tokenizers/tinystories-8k-500k"),
                               output_path=Path("data/processed/tinystories-full-8k"), *,
                               train_urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                               validation_urls: Sequence[str] = TINYSTORIES_VALIDATION_URLS,
                               progress: ProgressCallback | None = None) -> dict[str, Any]:
    dest = Path(output_path).resolve()
    if dest.exists() and not _target(dest):
        m = validate_tinystories_corpus(dest, tokenizer_path=tokenizer_path)
        pins = {"train": (TINYSTORIES_TRAIN_SHA256, TINYSTORIES_TRAIN_BYTES,
                          TINYSTORIES_TRAIN_STORIES),
                "validation": (TINYSTORIES_VALIDATION_SHA256, TINYSTORIES_VALIDATION_BYTES,
                               TINYSTORIES_VALIDATION_STORIES)}
        ok = all((m["sources"][n].get("sha256"), m["sources"][n].get("size_bytes"),
                  m["sources"][n].get("stories")) == p and
                 m["corpora"][n].get("documents") == p[2] for n, p in pins.items())
        if not ok or m["tokenizer"].get("vocab_size") != EXPECTED_VOCAB:
            raise FileExistsError("existing TinyStories corpus was built from different sources "
                                  "or counts")
        return {"command": "prepare-tinystories-corpus", "manifest": m, "output": str(dest),
                "reused": True}
    d = Path(data_dir)
    trs, vas = d / "TinyStories-train.txt", d / "TinyStories-valid.txt"
    trv = download_pinned_file(trs, urls=train_urls, expected_size=TINYSTORIES_TRAIN_BYTES,
                               expected_sha256=TINYSTORIES_TRAIN_SHA256, progress=progress)
    vav = download_pinned_file(vas, urls=validation_urls,
                               expected_size=TINYSTORIES_VALIDATION_BYTES,
                               expected_sha256=TINYSTORIES_VALIDATION_SHA256, progress=progress)
    return build_tinystories_corpus(trs, vas, tokenizer_path, output_path,
                                    train_verification=trv, validation_verification=vav,
                                    expected_train_stories=TINYSTORIES_TRAIN_STORIES,
                                    expected_validation_stories=TINYSTORIES_VALIDATION_STORIES,
                                    expected_vocab_size=EXPECTED_VOCAB)
