"""Text ingestion and the portable ``.pt`` token-corpus artifact.

A corpus is one flat token stream plus document offsets (``documents + 1``
entries, from 0 to the token count), the vocabulary size, the EOS id, the
tokenizer fingerprint and whether each document ends with an appended EOS.
Its content fingerprint is sha256 over a canonical JSON header followed by the
tokens and the offsets as little-endian int64 -- the same for the ``.pt`` and
the mmap container, so a checkpoint identifies data, not storage. Artifact
name ``nano_megatron.token_corpus`` v2 (v1 without the stored fingerprint, and
the two tensor-only legacy files, still load). Format and fingerprint recipe
follow the reference (src/nano_megatron/data/corpus.py:16-449) so corpora are
interchangeable.
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Iterable, Iterator
from pathlib import Path
from typing import Any

import torch

ARTIFACT_NAME = "nano_megatron.token_corpus"
ARTIFACT_VERSION = 2
_INT_DTYPES = (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64)
_KEYS_V1 = frozenset({"artifact", "format_version", "tokens", "document_offsets", "documents",
                      "vocab_size", "eos_id", "tokenizer_fingerprint", "append_eos"})
_KEYS_V2 = _KEYS_V1 | {"fingerprint"}


def corpus_fingerprint(*, append_eos: bool, documents: int, eos_id, tokenizer_fingerprint,
                       vocab_size: int, token_chunks: Iterable, offset_chunks: Iterable) -> str:
    header = {"append_eos": append_eos, "artifact": ARTIFACT_NAME, "documents": documents,
              "eos_id": eos_id, "format_version": ARTIFACT_VERSION,
              "tokenizer_fingerprint": tokenizer_fingerprint, "vocab_size": vocab_size}
    h = hashlib.sha256(json.dumps(header, ensure_ascii=False, sort_keys=True,
                                  separators=(",", ":")).encode("utf-8"))
    for c in token_chunks:
        h.update(c)
    for c in offset_chunks:
        h.update(c)
    return h.hexdigest()


def check_text_key(text_key: str) -> str:
    if not isinstance(text_key, str):
        raise TypeError("text_key must be a string")
    if not text_key.strip():
        raise ValueError("text_key must not be empty")
    return text_key


def _doc_text(text: Any, where: str) -> str:
    if not isinstance(text, str):
        raise TypeError(f"{where}: text must be a string")
    if not text.strip():
        raise ValueError(f"{where}: text must not be empty")
    return text


def iter_jsonl_text(path, *, text_key: str = "text") -> Iterator[str]:
    """Non-empty strings from a JSONL file; errors name file:line."""
    src = Path(path)
    key = check_text_key(text_key)
    n = 0
    with src.open("r", encoding="utf-8") as f:
        for lineno, line in enumerate(f, start=1):
            n += 1
            where = f"{src}:{lineno}"
            if not line.strip():
                raise ValueError(f"{where}: JSONL record must not be empty")
            try:
                rec = json.loads(line)
            except json.JSONDecodeError as e:
                raise ValueError(f"{where}: invalid JSON ({e.msg} at column {e.colno})") from e
            if not isinstance(rec, dict):
                raise TypeError(f"{where}: JSONL record must be an object")
            if key not in rec:
                raise ValueError(f"{where}: missing text key {key!r}")
            yield _doc_text(rec[key], f"{where}:{key}")
    if n == 0:
        raise ValueError(f"{src}:1: JSONL file must contain at least one record")


def check_tokenizer(tokenizer) -> tuple[int, int, str]:
    v, eos, fp = tokenizer.vocab_size, tokenizer.eos_token_id, tokenizer.fingerprint
    if isinstance(v, bool) or not isinstance(v, int) or v < 1:
        raise ValueError("tokenizer.vocab_size must be a positive integer")
    if isinstance(eos, bool) or not isinstance(eos, int):
        raise TypeError("tokenizer.eos_token_id must be an integer")
    if not 0 <= eos < v:
        raise ValueError("tokenizer.eos_token_id must be inside the tokenizer vocabulary")
    if not isinstance(fp, str) or not fp.strip():
        raise ValueError("tokenizer.fingerprint must be a non-empty string")
    return v, eos, fp


def check_token_ids(ids: Any, *, document: int, vocab_size: int) -> list[int]:
    if not isinstance(ids, list):
        raise TypeError(f"document {document}: tokenizer.encode() must return list[int]")
    if not ids:
        raise ValueError(f"document {document}: tokenizer produced no token ids")
    for off, t in enumerate(ids):
        if isinstance(t, bool) or not isinstance(t, int):
            raise TypeError(f"document {document}: token id at offset {off} must be an integer")
        if not 0 <= t < vocab_size:
            raise ValueError(f"document {document}: token id {t} at offset {off} is outside "
                             f"vocab_size={vocab_size}")
    return ids


def _i64_bytes(t: torch.Tensor) -> bytes:
    return t.numpy().astype("<i8", copy=False).tobytes(order="C")


class TokenCorpus:
    """A flat token stream plus the metadata that validates document boundaries."""

    __slots__ = ("tokens", "document_offsets", "documents", "vocab_size", "eos_id",
                 "tokenizer_fingerprint", "append_eos")

    def __init__(self, *, tokens: torch.Tensor, document_offsets: torch.Tensor, documents: int,
                 vocab_size: int, eos_id: int | None, tokenizer_fingerprint: str | None,
                 append_eos: bool) -> None:
        for name, t in (("tokens", tokens), ("document_offsets", document_offsets)):
            if not isinstance(t, torch.Tensor):
                raise TypeError(f"{name} must be a torch.Tensor")
            if t.ndim != 1:
                raise ValueError(f"{name} must be one-dimensional")
            if t.dtype not in _INT_DTYPES:
                raise TypeError(f"{name} must use an integer dtype")
            if t.device.type != "cpu":
                raise ValueError(f"{name} must reside on CPU")
        self.tokens = tokens.to(torch.long).contiguous()
        self.document_offsets = document_offsets.to(torch.long).contiguous()
        self.documents, self.vocab_size, self.eos_id = documents, vocab_size, eos_id
        self.tokenizer_fingerprint, self.append_eos = tokenizer_fingerprint, append_eos
        self._validate()

    def _validate(self) -> None:
        offs = self.document_offsets
        if isinstance(self.documents, bool) or not isinstance(self.documents, int):
            raise TypeError("documents must be an integer")
        if self.documents < 1:
            raise ValueError("documents must be positive")
        if offs.numel() != self.documents + 1:
            raise ValueError("document_offsets must contain documents + 1 entries")
        if int(offs[0]) != 0:
            raise ValueError("document_offsets must start at zero")
        if int(offs[-1]) != self.tokens.numel():
            raise ValueError("document_offsets must end at the token count")
        if not isinstance(self.append_eos, bool):
            raise TypeError("append_eos must be a boolean")
        diffs = offs[1:] - offs[:-1]
        if self.is_legacy:
            if self.documents != 1 or self.append_eos:
                raise ValueError("legacy token corpora must be one document without appended EOS")
            if bool((diffs < 0).any()):
                raise ValueError("legacy document_offsets must be non-decreasing")
        elif bool((diffs <= 0).any()):
            raise ValueError("structured token corpora cannot contain empty documents")
        if isinstance(self.vocab_size, bool) or not isinstance(self.vocab_size, int):
            raise TypeError("vocab_size must be an integer")
        if self.vocab_size < 1:
            raise ValueError("vocab_size must be positive")
        if self.tokens.numel() and (int(self.tokens.min()) < 0 or
                                    int(self.tokens.max()) >= self.vocab_size):
            raise ValueError("tokens contain ids outside vocab_size")
        if self.is_legacy:
            return
        if isinstance(self.eos_id, bool) or not isinstance(self.eos_id, int):
            raise TypeError("eos_id must be an integer")
        if not 0 <= self.eos_id < self.vocab_size:
            raise ValueError("eos_id must be inside vocab_size")
        if not isinstance(self.tokenizer_fingerprint, str) or \
                not self.tokenizer_fingerprint.strip():
            raise ValueError("tokenizer_fingerprint must be a non-empty string")
        if self.append_eos and not bool((self.tokens[offs[1:] - 1] == self.eos_id).all()):
            raise ValueError("every document must end with eos_id when append_eos is true")

    def __eq__(self, other: object) -> bool:
        if not isinstance(other, TokenCorpus):
            return NotImplemented
        return (torch.equal(self.tokens, other.tokens) and
                torch.equal(self.document_offsets, other.document_offsets) and
                (self.documents, self.vocab_size, self.eos_id, self.tokenizer_fingerprint,
                 self.append_eos) == (other.documents, other.vocab_size, other.eos_id,
                                      other.tokenizer_fingerprint, other.append_eos))

    __hash__ = None

    @property
    def is_legacy(self) -> bool:
        return self.eos_id is None and self.tokenizer_fingerprint is None

    @property
    def fingerprint(self) -> str:
        return corpus_fingerprint(append_eos=self.append_eos, documents=self.documents,
                                  eos_id=self.eos_id,
                                  tokenizer_fingerprint=self.tokenizer_fingerprint,
                                  vocab_size=self.vocab_size,
                                  token_chunks=(_i64_bytes(self.tokens),),
                                  offset_chunks=(_i64_bytes(self.document_offsets),))

    @classmethod
    def from_texts(cls, texts: Iterable[str], tokenizer, *, append_eos: bool = True
                   ) -> "TokenCorpus":
        if not isinstance(append_eos, bool):
            raise TypeError("append_eos must be a boolean")
        if isinstance(texts, (str, bytes)):
            raise TypeError("texts must be an iterable of documents, not one string")
        vocab, eos, fp = check_tokenizer(tokenizer)
        flat: list[int] = []
        offsets = [0]
        n = 0
        for n, text in enumerate(texts, start=1):
            ids = check_token_ids(tokenizer.encode(_doc_text(text, f"document {n}"),
                                                   add_bos=False, add_eos=False),
                                  document=n, vocab_size=vocab)
            flat.extend(ids)
            if append_eos:
                flat.append(eos)
            offsets.append(len(flat))
        if n == 0:
            raise ValueError("at least one document is required")
        return cls(tokens=torch.tensor(flat, dtype=torch.long),
                   document_offsets=torch.tensor(offsets, dtype=torch.long), documents=n,
                   vocab_size=vocab, eos_id=eos, tokenizer_fingerprint=fp, append_eos=append_eos)

    @classmethod
    def from_jsonl(cls, path, tokenizer, *, text_key: str = "text", append_eos: bool = True
                   ) -> "TokenCorpus":
        return cls.from_texts(iter_jsonl_text(path, text_key=text_key), tokenizer,
                              append_eos=append_eos)

    def save(self, path) -> None:
        if self.is_legacy:
            raise ValueError("legacy token tensors cannot be saved as structured corpora")
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        payload = {"artifact": ARTIFACT_NAME, "format_version": ARTIFACT_VERSION,
                   "tokens": self.tokens, "document_offsets": self.document_offsets,
                   "documents": self.documents, "vocab_size": self.vocab_size,
                   "eos_id": self.eos_id, "tokenizer_fingerprint": self.tokenizer_fingerprint,
                   "append_eos": self.append_eos, "fingerprint": self.fingerprint}
        try:
            f = target.open("xb")
        except FileExistsError as e:
            raise FileExistsError(f"refusing to overwrite token corpus: {target}") from e
        try:
            with f:
                torch.save(payload, f)
        except BaseException:
            target.unlink(missing_ok=True)
            raise

    @classmethod
    def load(cls, path) -> "TokenCorpus":
        v = torch.load(Path(path), map_location="cpu", weights_only=True)
        if isinstance(v, torch.Tensor):
            return cls._legacy(v)
        if not isinstance(v, dict):
            raise TypeError("token file must contain TokenCorpus data, a Tensor, or "
                            "{'tokens': Tensor}")
        if set(v) == {"tokens"}:
            if not isinstance(v["tokens"], torch.Tensor):
                raise TypeError("legacy {'tokens': ...} value must be a Tensor")
            return cls._legacy(v["tokens"])
        if v.get("artifact") != ARTIFACT_NAME:
            raise ValueError(f"unsupported token artifact: {v.get('artifact')!r}")
        ver = v.get("format_version")
        keys = {1: _KEYS_V1, ARTIFACT_VERSION: _KEYS_V2}.get(ver) \
            if isinstance(ver, int) and not isinstance(ver, bool) else None
        if keys is None:
            raise ValueError(f"unsupported TokenCorpus format_version: {ver!r}")
        if set(v) != keys:
            parts = []
            if keys - set(v):
                parts.append("missing keys: " + ", ".join(sorted(keys - set(v))))
            if set(v) - keys:
                parts.append("unknown keys: " + ", ".join(sorted(set(v) - keys)))
            raise ValueError("invalid TokenCorpus artifact (" + "; ".join(parts) + ")")
        c = cls(tokens=v["tokens"], document_offsets=v["document_offsets"],
                documents=v["documents"], vocab_size=v["vocab_size"], eos_id=v["eos_id"],
                tokenizer_fingerprint=v["tokenizer_fingerprint"], append_eos=v["append_eos"])
        if ver == ARTIFACT_VERSION:
            fp = v["fingerprint"]
            ok = isinstance(fp, str) and len(fp) == 64
            if ok:
                try:
                    bytes.fromhex(fp)
                except ValueError:
                    ok = False
            if not ok:
                raise ValueError("TokenCorpus fingerprint must be a SHA256 hex digest")
            if c.fingerprint != fp:
                raise ValueError("TokenCorpus content fingerprint does not match its payload")
        return c

    @classmethod
    def _legacy(cls, t: torch.Tensor) -> "TokenCorpus":
        if t.ndim != 1:
            raise ValueError("legacy tokens must be one-dimensional")
        if t.dtype not in _INT_DTYPES:
            raise TypeError("legacy tokens must use an integer dtype")
        t = t.to(torch.long).contiguous()
        if t.numel() and int(t.min()) < 0:
            raise ValueError("legacy tokens must be non-negative")
        return cls(tokens=t, document_offsets=torch.tensor([0, t.numel()]), documents=1,
                   vocab_size=int(t.max()) + 1 if t.numel() else 1, eos_id=None,
                   tokenizer_fingerprint=None, append_eos=False)


def build_token_corpus(texts: Iterable[str], tokenizer, *, append_eos: bool = True
                       ) -> TokenCorpus:
    return TokenCorpus.from_texts(texts, tokenizer, append_eos=append_eos)


def preprocess_jsonl(input_path, output_path, tokenizer, *, text_key: str = "text",
                     append_eos: bool = True) -> TokenCorpus:
    c = TokenCorpus.from_jsonl(input_path, tokenizer, text_key=text_key, append_eos=append_eos)
    c.save(output_path)
    return c
