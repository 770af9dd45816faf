"""The full TinyStories training artifact: train and validation memory-mapped corpora
under one manifest.

Directory layout (nothing else may be in it)::

    <output>/manifest.json     what was built, from what, with which tokenizer
    <output>/train.mmap/       MMapTokenCorpus of every train story (EOS appended)
    <output>/validation.mmap/  the same for the validation stories
    <output>/.complete         written last: a directory without it is unfinished

A build writes everything into a temporary sibling directory, validates it there and
renames it into place, so a reader never sees a half-written corpus; an existing corpus
is validated and reused only if its sources, counts and tokenizer are the ones asked for.
Validation reads every manifest field against the files it describes (sizes, digests,
fingerprints, tokenizer identity) and fails with :class:`TinyStoriesCorpusError` naming
the field. Manifest keys and the directory names are the reference's
(src/nano_megatron/data/tinystories_corpus.py), so a corpus built by either framework
trains the other.
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
SPLITS = ("train", "validation")
_REVISION = {"canonical": TINYSTORIES_CANONICAL_REVISION, "mirror": TINYSTORIES_MIRROR_REVISION}
_DELIM = TINYSTORIES_DELIMITER.decode("ascii")
_PINS = {"train": (TINYSTORIES_TRAIN_SHA256, TINYSTORIES_TRAIN_BYTES, TINYSTORIES_TRAIN_STORIES),
         "validation": (TINYSTORIES_VALIDATION_SHA256, TINYSTORIES_VALIDATION_BYTES,
                        TINYSTORIES_VALIDATION_STORIES)}


class TinyStoriesCorpusError(ValueError):
    """A TinyStories corpus directory does not match its manifest or the request."""


def _fail(field: str, problem: str):
    raise TinyStoriesCorpusError(f"TinyStories corpus: {field} {problem}")


class _Fields:
    """Typed reads of a manifest object; every failure names the dotted field."""

    def __init__(self, obj: Any, where: str, keys: set | None = None) -> None:
        if not isinstance(obj, Mapping):
            _fail(where, "must be a JSON object")
        if keys is not None and set(obj) != keys:
            _fail(where, f"has keys {sorted(obj)}, expected {sorted(keys)}")
        self.obj, self.where = obj, where

    def _name(self, key: str) -> str:
        return f"{self.where}.{key}" if self.where else key

    def text(self, key: str) -> str:
        v = self.obj.get(key)
        if not isinstance(v, str) or not v:
            _fail(self._name(key), "must be a non-empty string")
        return v

    def count(self, key: str, low: int = 1) -> int:
        v = self.obj.get(key)
        if isinstance(v, bool) or not isinstance(v, int) or v < low:
            _fail(self._name(key), f"must be an int >= {low}")
        return v

    def sub(self, key: str, keys: set | None = None) -> "_Fields":
        return _Fields(self.obj.get(key), self._name(key), keys)

    def equals(self, key: str, want: Any) -> None:
        if self.obj.get(key) != want:
            _fail(self._name(key), f"is {self.obj.get(key)!r}, expected {want!r}")


def _corpus_entry(directory: str, c: MMapTokenCorpus) -> dict[str, Any]:
    return {"append_eos": c.append_eos, "directory": directory,
            "document_offsets_sha256": c.document_offsets_sha256, "documents": c.documents,
            "fingerprint": c.fingerprint, "token_count": c.token_count,
            "token_dtype": c.token_dtype.str, "tokens_sha256": c.tokens_sha256}


def _source_entry(v: FileVerification, stories: int) -> dict[str, Any]:
    return {"path": str(v.path), "sha256": v.sha256, "size_bytes": v.size_bytes,
            "stories": stories, "story_delimiter": _DELIM}


def _open_split(root: Path, entry: _Fields) -> MMapTokenCorpus:
    rel = Path(entry.text("directory"))
    if rel.is_absolute() or ".." in rel.parts:
        _fail(entry._name("directory"), "must be a relative path inside the corpus")
    if not (root / rel).is_dir():
        _fail(entry._name("directory"), f"points at a missing directory {root / rel}")
    try:
        return MMapTokenCorpus.load(root / rel)
    except (OSError, ValueError) as e:
        raise TinyStoriesCorpusError(f"TinyStories corpus: {rel} does not load ({e})") from e


def _check_sources(m: _Fields) -> None:
    src = m.sub("sources", set(SPLITS))
    digests = []
    for split in SPLITS:
        s = src.sub(split, {"path", "sha256", "size_bytes", "stories", "story_delimiter"})
        s.text("path")
        dg = s.text("sha256")
        if len(dg) != 64 or any(c not in "0123456789abcdefABCDEF" for c in dg):
            _fail(s._name("sha256"), "is not a SHA-256 hex digest")
        s.count("size_bytes")
        s.count("stories")
        s.equals("story_delimiter", _DELIM)
        digests.append(dg)
    if digests[0] == digests[1]:
        _fail("sources", "name the same file for train and validation")


def validate_tinystories_corpus(path, *, tokenizer_path=None) -> dict[str, Any]:
    """The manifest of a complete, self-consistent corpus directory (with
    ``tokenizer_path``: built with exactly that tokenizer)."""
    root = Path(path).resolve()
    if not (root.is_dir() and (root / COMPLETE).is_file()):
        _fail(str(root), "is missing or unfinished (no .complete marker)")
    entries = {p.name for p in root.iterdir()}
    if entries != {COMPLETE, MANIFEST, TRAIN_DIR, VALIDATION_DIR}:
        _fail(str(root), f"holds {sorted(entries)}; expected exactly "
                         f"{sorted({COMPLETE, MANIFEST, TRAIN_DIR, VALIDATION_DIR})}")
    try:
        raw = json.loads((root / MANIFEST).read_text(encoding="utf-8"))
    except (OSError, UnicodeDecodeError, json.JSONDecodeError) as e:
        raise TinyStoriesCorpusError(f"TinyStories corpus: unreadable manifest ({e})") from e
    m = _Fields(raw, "", {"artifact", "corpora", "format_version", "source_revision",
                          "sources", "tokenizer"})
    m.equals("artifact", ARTIFACT_NAME)
    m.equals("format_version", ARTIFACT_VERSION)
    m.equals("source_revision", _REVISION)
    tok = m.sub("tokenizer", {"eos_token_id", "fingerprint", "path", "vocab_size"})
    fp = tok.text("fingerprint")
    tok.text("path")
    vocab = tok.count("vocab_size")
    eos = tok.count("eos_token_id", 0)
    if eos >= vocab:
        _fail("tokenizer.eos_token_id", f"{eos} is outside the vocabulary of {vocab}")
    if tokenizer_path is not None:
        t = ByteLevelBPETokenizer.load(tokenizer_path)
        if (t.fingerprint, t.vocab_size, t.eos_token_id) != (fp, vocab, eos):
            _fail("tokenizer", f"does not match the tokenizer at {tokenizer_path}")
    corpora = m.sub("corpora", set(SPLITS))
    opened: dict[str, MMapTokenCorpus] = {}
    try:
        for split in SPLITS:
            entry = corpora.sub(split)
            c = opened[split] = _open_split(root, entry)
            if dict(entry.obj) != _corpus_entry(str(entry.obj.get("directory")), c):
                _fail(f"corpora.{split}", "disagrees with the corpus files it describes")
            if not c.append_eos:
                _fail(f"corpora.{split}", "was built without EOS after each story")
            if (c.tokenizer_fingerprint, c.vocab_size, c.eos_id) != (fp, vocab, eos):
                _fail(f"corpora.{split}", "was tokenized by a different tokenizer")
        if opened["train"].fingerprint == opened["validation"].fingerprint:
            _fail("corpora", "hold the same corpus for train and validation")
    finally:
        for c in opened.values():
            c.close()
    _check_sources(m)
    return raw


def _empty_or_absent(d: Path) -> bool:
    """True for an empty directory (replaceable), False if absent; raises otherwise
    unless it is a non-empty directory (an existing corpus, returned as False too)."""
    if d.is_symlink():
        raise FileExistsError(f"{d} is a symlink; not replacing it")
    if not d.exists():
        return False
    if not d.is_dir():
        raise FileExistsError(f"{d} exists and is not a directory")
    return next(d.iterdir(), None) is None


def _reuse(dest: Path, tokenizer_path, matches) -> dict[str, Any]:
    m = validate_tinystories_corpus(dest, tokenizer_path=tokenizer_path)
    if not matches(m):
        raise FileExistsError(f"{dest} holds a TinyStories corpus built from other sources "
                              "or story counts")
    return {"command": "prepare-tinystories-corpus", "manifest": m, "output": str(dest),
            "reused": True}


def build_tinystories_corpus(train_source, validation_source, tokenizer_path, output_path, *,
                             train_verification: FileVerification,
                             validation_verification: FileVerification,
                             expected_train_stories: int, expected_validation_stories: int,
                             expected_vocab_size: int = EXPECTED_VOCAB) -> dict[str, Any]:
    """Tokenize both verified sources into ``output_path`` (or reuse a matching corpus)."""
    paths = {"train": Path(train_source).resolve(),
             "validation": Path(validation_source).resolve()}
    if paths["train"] == paths["validation"]:
        raise ValueError("train and validation sources are the same file")
    checks = {}
    for split, v in (("train", train_verification), ("validation", validation_verification)):
        if v.path.resolve() != paths[split]:
            raise ValueError(f"the {split} verification is for {v.path}, not {paths[split]}")
        checks[split] = verify_file(paths[split], expected_size=v.size_bytes,
                                    expected_sha256=v.sha256)
    if checks["train"].sha256 == checks["validation"].sha256:
        raise ValueError("train and validation sources have the same SHA-256")
    want_stories = {"train": expected_train_stories, "validation": expected_validation_stories}
    tok_path = Path(tokenizer_path).resolve()
    tok = ByteLevelBPETokenizer.load(tok_path)
    if tok.vocab_size != expected_vocab_size:
        raise ValueError(f"tokenizer at {tok_path} has {tok.vocab_size} tokens, expected "
                         f"{expected_vocab_size}")
    dest = Path(output_path).resolve()
    empty = _empty_or_absent(dest)
    if dest.exists() and not empty:
        return _reuse(dest, tok_path, lambda m: all(
            m["sources"][s] == _source_entry(checks[s], want_stories[s]) and
            m["corpora"][s].get("documents") == want_stories[s] for s in SPLITS))
    dest.parent.mkdir(parents=True, exist_ok=True)
    work = Path(tempfile.mkdtemp(prefix=f".{dest.name}.tmp-", dir=dest.parent))
    placeholder_removed = False
    try:
        built = {}
        for split, sub in (("train", TRAIN_DIR), ("validation", VALIDATION_DIR)):
            c = preprocess_texts_mmap(iter_delimited_stories(paths[split]), work / sub, tok)
            if c.documents != want_stories[split]:
                raise TinyStoriesCorpusError(f"TinyStories corpus: {split} source yielded "
                                             f"{c.documents} stories, expected "
                                             f"{want_stories[split]}")
            built[split] = (sub, c)
        manifest = {
            "artifact": ARTIFACT_NAME, "format_version": ARTIFACT_VERSION,
            "corpora": {s: _corpus_entry(sub, c) for s, (sub, c) in built.items()},
            "source_revision": dict(_REVISION),
            "sources": {s: _source_entry(checks[s], c.documents) for s, (_, c) in built.items()},
            "tokenizer": {"eos_token_id": tok.eos_token_id, "fingerprint": tok.fingerprint,
                          "path": str(tok_path), "vocab_size": tok.vocab_size}}
        (work / MANIFEST).write_text(json.dumps(manifest, ensure_ascii=False, indent=2,
                                                sort_keys=True) + "\n", encoding="utf-8")
        (work / COMPLETE).write_text("complete\n", encoding="utf-8")
        validate_tinystories_corpus(work, tokenizer_path=tok_path)
        if empty:
            dest.rmdir()
            placeholder_removed = True
        elif dest.exists() or dest.is_symlink():
            raise FileExistsError(f"{dest} appeared while the corpus was being built")
        os.replace(work, dest)
    except BaseException:
        if placeholder_removed and not dest.exists():
            dest.mkdir()
        raise
    finally:
        if work.exists():
            shutil.rmtree(work)
    return {"command": "prepare-tinystories-corpus",
            "manifest": validate_tinystories_corpus(dest, tokenizer_path=tok_path),
            "output": str(dest), "reused": False}


def prepare_tinystories_corpus(data_dir=Path("data/raw/tinystories"),
                               tokenizer_path=Path("data/tokenizers/tinystories-8k-500k"),
                               output_path=Path("data/processed/tinystories-full-8k"), *,
                               train_urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                               validation_urls: Sequence[str] = TINYSTORIES_VALIDATION_URLS,
                               progress: ProgressCallback | None = None) -> dict[str, Any]:
    """Download both pinned files into ``data_dir`` and build the corpus (or reuse one that
    was built from exactly the pinned files)."""
    dest = Path(output_path).resolve()
    if dest.exists() and not _empty_or_absent(dest):
        def pinned(m) -> bool:
            ok = all((m["sources"][s].get("sha256"), m["sources"][s].get("size_bytes"),
                      m["sources"][s].get("stories")) == _PINS[s] and
                     m["corpora"][s].get("documents") == _PINS[s][2] for s in SPLITS)
            return ok and m["tokenizer"].get("vocab_size") == EXPECTED_VOCAB
        return _reuse(dest, tokenizer_path, pinned)
    d = Path(data_dir)
    files = {"train": d / "TinyStories-train.txt", "validation": d / "TinyStories-valid.txt"}
    urls = {"train": train_urls, "validation": validation_urls}
    got = {s: download_pinned_file(files[s], urls=urls[s], expected_size=_PINS[s][1],
                                   expected_sha256=_PINS[s][0], progress=progress)
           for s in SPLITS}
    return build_tinystories_corpus(files["train"], files["validation"], tokenizer_path,
                                    output_path, train_verification=got["train"],
                                    validation_verification=got["validation"],
                                    expected_train_stories=TINYSTORIES_TRAIN_STORIES,
                                    expected_validation_stories=TINYSTORIES_VALIDATION_STORIES,
                                    expected_vocab_size=EXPECTED_VOCAB)
