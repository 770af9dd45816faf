"""Read-only memory-mapped token corpus: ``tokens.bin`` + ``document_offsets.bin`` + ``metadata.json``.

Tokens are stored in the narrowest canonical little-endian unsigned type for
the vocabulary (``<u2`` up to 65,536 ids, else ``<u4``), offsets as ``<u8``.
The metadata records both files' sha256 and the container-independent logical
fingerprint shared with the ``.pt`` corpus. Writing streams documents in
batches into a temporary sibling directory, re-validates it, then renames it
into place. The on-disk layout and metadata keys follow the reference
(src/nano_megatron/data/mmap_corpus.py:25-616) so artifacts are interchangeable;
the read path here is the native ``TokenSource`` (C++ mmap + widening gather).
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from collections.abc import Iterable, Iterator
from pathlib import Path
from typing import Any

import numpy as np

from .corpus import check_token_ids, check_tokenizer, corpus_fingerprint, iter_jsonl_text

ARTIFACT_NAME = "nano_megatron.mmap_token_corpus"
ARTIFACT_VERSION = 1
TOKENS_FILE = "tokens.bin"
OFFSETS_FILE = "document_offsets.bin"
METADATA_FILE = "metadata.json"
OFFSET_DTYPE = np.dtype("<u8")
_SCAN = 1 << 20
_KEYS = frozenset({"append_eos", "artifact", "document_offsets_dtype", "document_offsets_sha256",
                   "documents", "eos_id", "fingerprint", "format_version", "token_count",
                   "token_dtype", "tokenizer_fingerprint", "tokens_sha256", "vocab_size"})


class MMapCorpusError(ValueError):
    """An mmap corpus exists but violates its artifact contract."""


def token_dtype_for_vocab(vocab_size: int) -> np.dtype:
    if vocab_size <= 1 << 16:
        return np.dtype("<u2")
    if vocab_size <= 1 << 32:
        return np.dtype("<u4")
    raise ValueError(f"mmap token corpora support vocab_size <= {1 << 32}, got {vocab_size}")


def _file_id(p: Path) -> tuple[int, int, int, int]:
    s = p.stat()
    return (s.st_dev, s.st_ino, s.st_size, s.st_mtime_ns)


def _int_field(meta: dict, key: str, lo: int, hi: int | None = None) -> int:
    v = meta.get(key)
    if isinstance(v, bool) or not isinstance(v, int):
        raise MMapCorpusError(f"mmap metadata field {key!r} must be an integer")
    if v < lo or (hi is not None and v > hi):
        rng = f">= {lo}" if hi is None else f"between {lo} and {hi}"
        raise MMapCorpusError(f"mmap metadata field {key!r} must be {rng}")
    return v


def _str_field(meta: dict, key: str) -> str:
    v = meta.get(key)
    if not isinstance(v, str) or not v.strip():
        raise MMapCorpusError(f"mmap metadata field {key!r} must be a non-empty string")
    return v


def _sha_field(meta: dict, key: str) -> str:
    v = _str_field(meta, key)
    try:
        ok = len(v) == 64 and bytes.fromhex(v) is not None
    except ValueError:
        ok = False
    if not ok:
        raise MMapCorpusError(f"mmap metadata field {key!r} must be a SHA256 hex digest")
    return v


class MMapTokenCorpus:
    """Validated metadata plus a lazily opened read-only view of ``tokens.bin``.

    The offsets index lives in ordinary memory; the token payload is opened on
    first access (never pickled, so worker processes reopen it themselves).
    """

    def __init__(self, *, path: Path, token_dtype: np.dtype, token_count: int,
                 document_offsets: np.ndarray, documents: int, vocab_size: int, eos_id: int,
                 tokenizer_fingerprint: str, append_eos: bool, tokens_sha256: str,
                 document_offsets_sha256: str, fingerprint: str, token_file_identity) -> None:
        self.path = path
        self.token_dtype = token_dtype
        self.token_count = token_count
        document_offsets.flags.writeable = False
        self.document_offsets = document_offsets
        self.documents = documents
        self.vocab_size = vocab_size
        self.eos_id = eos_id
        self.tokenizer_fingerprint = tokenizer_fingerprint
        self.append_eos = append_eos
        self.tokens_sha256 = tokens_sha256
        self.document_offsets_sha256 = document_offsets_sha256
        self.fingerprint = fingerprint
        self._identity = token_file_identity
        self._tokens = None
        self._source = None

    is_legacy = property(lambda self: False)

    def _check_identity(self) -> None:
        if _file_id(self.path / TOKENS_FILE) != self._identity:
            raise MMapCorpusError("tokens.bin changed after the mmap corpus was validated; "
                                  "reload the artifact")

    @property
    def tokens(self) -> np.memmap:
        if self._tokens is None:
            self._check_identity()
            t = np.memmap(self.path / TOKENS_FILE, dtype=self.token_dtype, mode="r",
                          shape=(self.token_count,))
            t.flags.writeable = False
            self._tokens = t
        return self._tokens

    def native_source(self):
        """The C++ ``TokenSource`` over ``tokens.bin`` (mmap + widening window gather)."""
        if self._source is None:
            from nano_megatron_b200.native import native

            self._check_identity()
            self._source = native().TokenSource(str(self.path / TOKENS_FILE),
                                                self.token_dtype.itemsize, self.token_count)
        return self._source

    def read_tokens(self, start: int, stop: int) -> np.ndarray:
        for name, v in (("start", start), ("stop", stop)):
            if isinstance(v, bool) or not isinstance(v, int):
                raise TypeError(f"{name} must be an integer")
        if start < 0 or stop < start or stop > self.token_count:
            raise IndexError(f"invalid token range [{start}, {stop}) for "
                             f"token_count={self.token_count}")
        return self.tokens[start:stop]

    def close(self) -> None:
        self._tokens = None
        self._source = None

    def __len__(self) -> int:
        return self.token_count

    def __getstate__(self) -> dict[str, Any]:
        s = self.__dict__.copy()
        s["_tokens"] = None
        s["_source"] = None
        return s

    def __setstate__(self, s: dict[str, Any]) -> None:
        self.__dict__.update(s)
        self.document_offsets.flags.writeable = False

    @classmethod
    def load(cls, path) -> "MMapTokenCorpus":
        d = Path(path).resolve()
        if not d.exists():
            raise FileNotFoundError(f"mmap corpus directory does not exist: {d}")
        if not d.is_dir():
            raise NotADirectoryError(f"mmap corpus path is not a directory: {d}")
        want = {TOKENS_FILE, OFFSETS_FILE, METADATA_FILE}
        have = {e.name for e in d.iterdir()}
        if have != want:
            parts = (["missing files: " + ", ".join(sorted(want - have))] if want - have else []) \
                + (["unknown files: " + ", ".join(sorted(have - want))] if have - want else [])
            raise MMapCorpusError("invalid mmap corpus directory (" + "; ".join(parts) + ")")
        for n in sorted(want):
            if (d / n).is_symlink() or not (d / n).is_file():
                raise MMapCorpusError(f"mmap corpus sidecar must be a regular file: {d / n}")
        try:
            meta = json.loads((d / METADATA_FILE).read_text(encoding="utf-8"))
        except (OSError, UnicodeDecodeError, json.JSONDecodeError) as e:
            raise MMapCorpusError(f"could not read mmap corpus metadata {d / METADATA_FILE}: "
                                  f"{e}") from e
        if not isinstance(meta, dict):
            raise MMapCorpusError("mmap corpus metadata must contain a JSON object")
        if set(meta) != _KEYS:
            parts = (["missing keys: " + ", ".join(sorted(_KEYS - set(meta)))]
                     if _KEYS - set(meta) else []) + \
                (["unknown keys: " + ", ".join(sorted(set(meta) - _KEYS))]
                 if set(meta) - _KEYS else [])
            raise MMapCorpusError("invalid mmap corpus metadata (" + "; ".join(parts) + ")")
        if meta.get("artifact") != ARTIFACT_NAME:
            raise MMapCorpusError(f"unsupported mmap corpus artifact: {meta.get('artifact')!r}")
        ver = _int_field(meta, "format_version", 1)
        if ver != ARTIFACT_VERSION:
            raise MMapCorpusError(f"unsupported mmap corpus format_version {ver}; expected "
                                  f"{ARTIFACT_VERSION}")
        vocab = _int_field(meta, "vocab_size", 1, 1 << 32)
        dt = token_dtype_for_vocab(vocab)
        if _str_field(meta, "token_dtype") != dt.str:
            raise MMapCorpusError("mmap token dtype is not the canonical dtype for vocab_size: "
                                  f"{meta['token_dtype']!r} != {dt.str!r}")
        if meta.get("document_offsets_dtype") != OFFSET_DTYPE.str:
            raise MMapCorpusError(f"document_offsets_dtype must be {OFFSET_DTYPE.str!r}")
        count = _int_field(meta, "token_count", 1, np.iinfo(np.int64).max)
        docs = _int_field(meta, "documents", 1, count)
        eos = _int_field(meta, "eos_id", 0, vocab - 1)
        tok_fp = _str_field(meta, "tokenizer_fingerprint")
        append = meta.get("append_eos")
        if not isinstance(append, bool):
            raise MMapCorpusError("mmap metadata field 'append_eos' must be a boolean")
        tok_sha, off_sha = _sha_field(meta, "tokens_sha256"), \
            _sha_field(meta, "document_offsets_sha256")
        want_fp = _sha_field(meta, "fingerprint")
        tpath, opath = d / TOKENS_FILE, d / OFFSETS_FILE
        ident = _file_id(tpath)
        if tpath.stat().st_size != count * dt.itemsize:
            raise MMapCorpusError("tokens.bin size does not match token_count and token_dtype: "
                                  f"{tpath.stat().st_size} != {count * dt.itemsize}")
        if opath.stat().st_size != (docs + 1) * OFFSET_DTYPE.itemsize:
            raise MMapCorpusError("document_offsets.bin size does not match documents: "
                                  f"{opath.stat().st_size} != "
                                  f"{(docs + 1) * OFFSET_DTYPE.itemsize}")
        offs = np.fromfile(opath, dtype=OFFSET_DTYPE)
        obytes = memoryview(offs).cast("B")
        if hashlib.sha256(obytes).hexdigest() != off_sha:
            raise MMapCorpusError("document_offsets.bin SHA256 does not match mmap metadata")
        if int(offs[0]) != 0:
            raise MMapCorpusError("document offsets must start at zero")
        if int(offs[-1]) != count:
            raise MMapCorpusError("document offsets must end at token_count")
        if np.any(offs[1:] <= offs[:-1]):
            raise MMapCorpusError("mmap token corpus cannot contain empty documents")
        toks = np.memmap(tpath, dtype=dt, mode="r", shape=(count,))
        try:
            digest = hashlib.sha256()
            top = 0

            def chunks() -> Iterator[bytes]:
                nonlocal top
                for s in range(0, count, _SCAN):
                    c = toks[s:s + _SCAN]
                    digest.update(c.tobytes(order="C"))
                    top = max(top, int(c.max()))
                    yield np.asarray(c, dtype="<i8").tobytes(order="C")

            fp = corpus_fingerprint(append_eos=append, documents=docs, eos_id=eos,
                                    tokenizer_fingerprint=tok_fp, vocab_size=vocab,
                                    token_chunks=chunks(), offset_chunks=(obytes,))
            if digest.hexdigest() != tok_sha:
                raise MMapCorpusError("tokens.bin SHA256 does not match mmap metadata")
            if top >= vocab:
                raise MMapCorpusError(f"tokens.bin contains token id {top} outside vocab_size")
            if append:
                ends = (offs[1:] - np.uint64(1)).astype(np.int64)
                for s in range(0, docs, _SCAN):
                    if np.any(toks[ends[s:s + _SCAN]] != eos):
                        raise MMapCorpusError("every document must end with eos_id when "
                                              "append_eos is true")
        finally:
            toks._mmap.close()
        if fp != want_fp:
            raise MMapCorpusError("mmap corpus logical fingerprint does not match its payload")
        if _file_id(tpath) != ident:
            raise MMapCorpusError("tokens.bin changed while the mmap corpus was being validated")
        return cls(path=d, token_dtype=dt, token_count=count, document_offsets=offs,
                   documents=docs, vocab_size=vocab, eos_id=eos, tokenizer_fingerprint=tok_fp,
                   append_eos=append, tokens_sha256=tok_sha, document_offsets_sha256=off_sha,
                   fingerprint=fp, token_file_identity=ident)


def _check_target(d: Path) -> bool:
    if d.is_symlink():
        raise FileExistsError(f"refusing to replace mmap corpus symlink: {d}")
    if not d.exists():
        return False
    if not d.is_dir():
        raise FileExistsError(f"mmap corpus path already exists: {d}")
    if any(d.iterdir()):
        raise FileExistsError(f"refusing to overwrite non-empty mmap corpus directory: {d}")
    return True


def preprocess_texts_mmap(texts: Iterable[str], output_path, tokenizer, *,
                          append_eos: bool = True, encoding_batch_size: int = 1024
                          ) -> MMapTokenCorpus:
    """Stream documents into an atomically published mmap artifact."""
    if not isinstance(append_eos, bool):
        raise TypeError("append_eos must be a boolean")
    if isinstance(encoding_batch_size, bool) or not isinstance(encoding_batch_size, int) or \
            encoding_batch_size < 1:
        raise ValueError("encoding_batch_size must be a positive integer")
    vocab, eos, tok_fp = check_tokenizer(tokenizer)
    dt = token_dtype_for_vocab(vocab)
    dest = Path(output_path)
    was_empty = _check_target(dest)
    dest.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=f".{dest.name}.tmp-", dir=dest.parent))
    removed = False
    try:
        tsha, osha = hashlib.sha256(), hashlib.sha256()
        count = docs = 0
        with (tmp / TOKENS_FILE).open("xb") as tf, (tmp / OFFSETS_FILE).open("xb") as of:
            zero = np.zeros(1, dtype=OFFSET_DTYPE).tobytes()
            of.write(zero)
            osha.update(zero)
            it = iter(texts)
            while True:
                batch = []
                for text in it:
                    if not isinstance(text, str):
                        raise TypeError(f"mmap document {docs + len(batch) + 1} must be a "
                                        f"string, got {type(text).__name__}")
                    batch.append(text)
                    if len(batch) == encoding_batch_size:
                        break
                if not batch:
                    break
                enc = getattr(tokenizer, "encode_batch", None)
                ids_list = enc(batch, add_bos=False, add_eos=False) if callable(enc) else \
                    [tokenizer.encode(t, add_bos=False, add_eos=False) for t in batch]
                if len(ids_list) != len(batch):
                    raise ValueError("tokenizer.encode_batch returned a different number of "
                                     "documents")
                ends = []
                parts = []
                for ids in ids_list:
                    docs += 1
                    ids = check_token_ids(ids, document=docs, vocab_size=vocab)
                    parts.append(np.asarray(ids + ([eos] if append_eos else []), dtype=dt))
                    count += len(parts[-1])
                    ends.append(count)
                blob = np.concatenate(parts).tobytes(order="C")
                tf.write(blob)
                tsha.update(blob)
                ob = np.asarray(ends, dtype=OFFSET_DTYPE).tobytes(order="C")
                of.write(ob)
                osha.update(ob)
                if len(batch) < encoding_batch_size:
                    break
        if docs == 0:
            raise ValueError("cannot build an mmap corpus from zero documents")
        offs = np.fromfile(tmp / OFFSETS_FILE, dtype=OFFSET_DTYPE)
        toks = np.memmap(tmp / TOKENS_FILE, dtype=dt, mode="r", shape=(count,))
        try:
            fp = corpus_fingerprint(
                append_eos=append_eos, documents=docs, eos_id=eos, tokenizer_fingerprint=tok_fp,
                vocab_size=vocab, token_chunks=(np.asarray(toks[s:s + _SCAN], dtype="<i8")
                                                .tobytes() for s in range(0, count, _SCAN)),
                offset_chunks=(memoryview(offs).cast("B"),))
        finally:
            toks._mmap.close()
        meta = {"append_eos": append_eos, "artifact": ARTIFACT_NAME,
                "document_offsets_dtype": OFFSET_DTYPE.str,
                "document_offsets_sha256": osha.hexdigest(), "documents": docs, "eos_id": eos,
                "fingerprint": fp, "format_version": ARTIFACT_VERSION, "token_count": count,
                "token_dtype": dt.str, "tokenizer_fingerprint": tok_fp,
                "tokens_sha256": tsha.hexdigest(), "vocab_size": vocab}
        (tmp / METADATA_FILE).write_text(json.dumps(meta, ensure_ascii=False, indent=2,
                                                    sort_keys=True) + "\n", encoding="utf-8")
        checked = MMapTokenCorpus.load(tmp)
        checked.close()
        if checked.fingerprint != fp:
            raise MMapCorpusError("mmap corpus fingerprint changed during self-validation")
        if was_empty:
            dest.rmdir()
            removed = True
        elif dest.exists() or dest.is_symlink():
            raise FileExistsError(f"mmap corpus path already exists: {dest}")
        os.replace(tmp, dest)
        checked.path = dest.resolve()
        checked._identity = _file_id(checked.path / TOKENS_FILE)
    except BaseException:
        if removed and not dest.exists():
            dest.mkdir()
        raise
    finally:
        if tmp.exists():
            shutil.rmtree(tmp)
    return checked


def preprocess_jsonl_mmap(input_path, output_path, tokenizer, *, text_key: str = "text",
                          append_eos: bool = True) -> MMapTokenCorpus:
    return preprocess_texts_mmap(iter_jsonl_text(input_path, text_key=text_key), output_path,
                                 tokenizer, append_eos=append_eos)
