"""Token corpora: text -> one flat token stream with document boundaries, and its ``.pt``
container.

A corpus is the concatenation of its documents' token ids (each optionally followed by
the EOS id) plus ``documents + 1`` offsets into that stream (``0 .. len(tokens)``), and
metadata: vocabulary size, EOS id, the tokenizer's fingerprint and whether EOS was
appended. Its identity is a content hash, independent of the container::

    sha256( canonical JSON of {append_eos, artifact, documents, eos_id, format_version,
                               tokenizer_fingerprint, vocab_size}
            || tokens as little-endian int64 || offsets as little-endian int64 )

so the ``.pt`` file and the memory-mapped directory (:mod:`.mmap_corpus`) of the same
corpus share one fingerprint and a checkpoint names data, not files. The ``.pt`` artifact
is a dict (``artifact = "nano_megatron.token_corpus"``, ``format_version`` 2 with the
stored ``fingerprint``; version 1 without it still loads) and two legacy forms still load
as a one-document corpus: a bare integer tensor and ``{"tokens": tensor}``. The artifact
keys and the hash recipe are the reference's (src/nano_megatron/data/corpus.py), so
corpora move between the frameworks.
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Iterable, Iterator
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

import torch

ARTIFACT_NAME = "nano_megatron.token_corpus"
ARTIFACT_VERSION = 2
_INT_DTYPES = (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64)
_PAYLOAD = ("tokens", "document_offsets")
_META = ("documents", "vocab_size", "eos_id", "tokenizer_fingerprint", "append_eos")
_KEYS_BY_VERSION = {1: frozenset(("artifact", "format_version") + _PAYLOAD + _META)}
_KEYS_BY_VERSION[2] = _KEYS_BY_VERSION[1] | {"fingerprint"}


def _is_int(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def corpus_fingerprint(*, append_eos: bool, documents: int, eos_id, tokenizer_fingerprint,
                       vocab_size: int, token_chunks: Iterable, offset_chunks: Iterable) -> str:
    """Content hash of a corpus whose int64 little-endian token and offset bytes arrive in
    chunks (so a memory-mapped corpus can be hashed without loading it)."""
    header = dict(append_eos=append_eos, artifact=ARTIFACT_NAME, documents=documents,
                  eos_id=eos_id, format_version=ARTIFACT_VERSION,
                  tokenizer_fingerprint=tokenizer_fingerprint, vocab_size=vocab_size)
    canon = json.dumps(header, sort_keys=True, separators=(",", ":"), ensure_ascii=False)
    h = hashlib.sha256(canon.encode("utf-8"))
    for chunk in (*token_chunks, *offset_chunks):
        h.update(chunk)
    return h.hexdigest()


# ---------------------------------------------------------------------- text input
def check_text_key(text_key: str) -> str:
    if not isinstance(text_key, str) or not text_key.strip():
        raise (TypeError if not isinstance(text_key, str) else ValueError)(
            f"text_key must be a non-blank string, got {text_key!r}")
    return text_key


def _document(text: Any, where: str) -> str:
    if not isinstance(text, str):
        raise TypeError(f"{where}: expected text, got {type(text).__name__}")
    if not text.strip():
        raise ValueError(f"{where}: the document is blank")
    return text


def iter_jsonl_text(path, *, text_key: str = "text") -> Iterator[str]:
    """The ``text_key`` string of every line of a JSONL file (one JSON object per line;
    blank lines, other JSON values, missing keys and blank texts are errors that name the
    file and line)."""
    src, key = Path(path), check_text_key(text_key)
    seen = False
    with src.open("r", encoding="utf-8") as f:
        for n, line in enumerate(f, start=1):
            seen = True
            at = f"{src}:{n}"
            if not line.strip():
                raise ValueError(f"{at}: blank line (every line must hold one JSON object)")
            try:
                obj = json.loads(line)
            except json.JSONDecodeError as e:
                raise ValueError(f"{at}: not valid JSON ({e.msg}, column {e.colno})") from e
            if not isinstance(obj, dict):
                raise TypeError(f"{at}: expected a JSON object, got {type(obj).__name__}")
            if key not in obj:
                raise ValueError(f"{at}: no {key!r} field")
            yield _document(obj[key], f"{at}:{key}")
    if not seen:
        raise ValueError(f"{src}: the JSONL file has no records")


def check_tokenizer(tokenizer) -> tuple[int, int, str]:
    """(vocab size, EOS id, fingerprint) of a tokenizer, checked for use in a corpus."""
    vocab, eos, fp = tokenizer.vocab_size, tokenizer.eos_token_id, tokenizer.fingerprint
    if not _is_int(vocab) or vocab < 1:
        raise ValueError(f"tokenizer vocab_size {vocab!r} is not an int >= 1")
    if not _is_int(eos):
        raise TypeError(f"tokenizer eos_token_id {eos!r} is not an int")
    if eos < 0 or eos >= vocab:
        raise ValueError(f"tokenizer eos_token_id {eos} lies outside its vocabulary [0, {vocab})")
    if not isinstance(fp, str) or not fp.strip():
        raise ValueError("the tokenizer has no fingerprint")
    return vocab, eos, fp


def check_token_ids(ids: Any, *, document: int, vocab_size: int) -> list[int]:
    """A document's encoding: a non-empty list of ints in ``[0, vocab_size)``."""
    if not isinstance(ids, list):
        raise TypeError(f"document {document}: encode() returned {type(ids).__name__}, "
                        "expected list[int]")
    if not ids:
        raise ValueError(f"document {document}: encodes to zero tokens")
    for pos, t in enumerate(ids):
        if not _is_int(t):
            raise TypeError(f"document {document}, token {pos}: {t!r} is not an int")
        if t < 0 or t >= vocab_size:
            raise ValueError(f"document {document}, token {pos}: id {t} is not in "
                             f"[0, {vocab_size})")
    return ids


def _le_int64(t: torch.Tensor) -> bytes:
    return t.numpy().astype("<i8", copy=False).tobytes(order="C")


def _as_int_vector(name: str, t: Any) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype not in _INT_DTYPES:
        raise TypeError(f"{name} has dtype {t.dtype}; an integer dtype is required")
    if t.ndim != 1 or t.device.type != "cpu":
        raise ValueError(f"{name} must be a 1-D CPU tensor (got {t.ndim}-D on {t.device})")
    return t.to(torch.long).contiguous()


@dataclass(frozen=True)
class _Meta:
    documents: int
    vocab_size: int
    eos_id: int | None
    tokenizer_fingerprint: str | None
    append_eos: bool

    @property
    def legacy(self) -> bool:
        return self.eos_id is None and self.tokenizer_fingerprint is None

    def check_scalars(self) -> None:
        if not _is_int(self.documents):
            raise TypeError(f"documents must be an int, got {self.documents!r}")
        if self.documents < 1:
            raise ValueError(f"a corpus needs at least one document, got {self.documents}")
        if not isinstance(self.append_eos, bool):
            raise TypeError(f"append_eos must be a bool, got {self.append_eos!r}")
        if not _is_int(self.vocab_size):
            raise TypeError(f"vocab_size must be an int, got {self.vocab_size!r}")
        if self.vocab_size < 1:
            raise ValueError(f"vocab_size must be >= 1, got {self.vocab_size}")
        if self.legacy:
            if self.documents != 1 or self.append_eos:
                raise ValueError("a legacy (tensor-only) corpus is one document without EOS")
            return
        if not _is_int(self.eos_id):
            raise TypeError(f"eos_id must be an int, got {self.eos_id!r}")
        if not 0 <= self.eos_id < self.vocab_size:
            raise ValueError(f"eos_id {self.eos_id} is not in [0, {self.vocab_size})")
        fp = self.tokenizer_fingerprint
        if not isinstance(fp, str) or not fp.strip():
            raise ValueError("tokenizer_fingerprint must be a non-blank string")


class TokenCorpus:
    """A flat token stream, its document offsets and the metadata that checks them."""

    __slots__ = ("tokens", "document_offsets", "documents", "vocab_size", "eos_id",
                 "tokenizer_fingerprint", "append_eos")

    def __init__(self, *, tokens: torch.Tensor, document_offsets: torch.Tensor, documents: int,
                 vocab_size: int, eos_id: int | None, tokenizer_fingerprint: str | None,
                 append_eos: bool) -> None:
        self.tokens = _as_int_vector("tokens", tokens)
        self.document_offsets = _as_int_vector("document_offsets", document_offsets)
        meta = _Meta(documents, vocab_size, eos_id, tokenizer_fingerprint, append_eos)
        for k, v in asdict(meta).items():
            setattr(self, k, v)
        meta.check_scalars()
        self._check_stream(meta)

    def _meta(self) -> _Meta:
        return _Meta(*(getattr(self, k) for k in _META))

    def _check_stream(self, meta: _Meta) -> None:
        offs, n = self.document_offsets, self.tokens.numel()
        if offs.numel() != meta.documents + 1:
            raise ValueError(f"{meta.documents} documents need {meta.documents + 1} offsets, "
                             f"got {offs.numel()}")
        if int(offs[0]) != 0 or int(offs[-1]) != n:
            raise ValueError(f"offsets must run from 0 to the token count {n}, got "
                             f"{int(offs[0])}..{int(offs[-1])}")
        lengths = offs[1:] - offs[:-1]
        if meta.legacy and bool((lengths < 0).any()):
            raise ValueError("legacy document offsets go backwards")
        if not meta.legacy and bool((lengths <= 0).any()):
            raise ValueError("empty documents are not allowed in a structured corpus")
        if n and not (0 <= int(self.tokens.min()) and int(self.tokens.max()) < meta.vocab_size):
            raise ValueError(f"tokens contain ids outside [0, vocab_size={meta.vocab_size})")
        if meta.append_eos and not bool((self.tokens[offs[1:] - 1] == meta.eos_id).all()):
            raise ValueError(f"append_eos is set but a document does not end with eos_id "
                             f"{meta.eos_id}")

    def __eq__(self, other: object) -> bool:
        if not isinstance(other, TokenCorpus):
            return NotImplemented
        return self._meta() == other._meta() and all(
            torch.equal(getattr(self, k), getattr(other, k)) for k in _PAYLOAD)

    __hash__ = None

    @property
    def is_legacy(self) -> bool:
        return self._meta().legacy

    @property
    def fingerprint(self) -> str:
        return corpus_fingerprint(append_eos=self.append_eos, documents=self.documents,
                                  eos_id=self.eos_id,
                                  tokenizer_fingerprint=self.tokenizer_fingerprint,
                                  vocab_size=self.vocab_size,
                                  token_chunks=[_le_int64(self.tokens)],
                                  offset_chunks=[_le_int64(self.document_offsets)])

    # ------------------------------------------------------------------ building
    @classmethod
    def from_texts(cls, texts: Iterable[str], tokenizer, *, append_eos: bool = True
                   ) -> "TokenCorpus":
        """Encode documents (no BOS/EOS from the tokenizer; EOS appended if asked)."""
        if not isinstance(append_eos, bool):
            raise TypeError(f"append_eos must be a bool, got {append_eos!r}")
        if isinstance(texts, (str, bytes)):
            raise TypeError("texts must be an iterable of documents; got a single string")
        vocab, eos, fp = check_tokenizer(tokenizer)
        stream: list[int] = []
        bounds = [0]
        for n, text in enumerate(texts, start=1):
            ids = tokenizer.encode(_document(text, f"document {n}"), add_bos=False,
                                   add_eos=False)
            stream += check_token_ids(ids, document=n, vocab_size=vocab)
            if append_eos:
                stream.append(eos)
            bounds.append(len(stream))
        if len(bounds) == 1:
            raise ValueError("no documents to build a corpus from")
        return cls(tokens=torch.tensor(stream, dtype=torch.long),
                   document_offsets=torch.tensor(bounds, dtype=torch.long),
                   documents=len(bounds) - 1, vocab_size=vocab, eos_id=eos,
                   tokenizer_fingerprint=fp, append_eos=append_eos)

    @classmethod
    def from_jsonl(cls, path, tokenizer, *, text_key: str = "text", append_eos: bool = True
                   ) -> "TokenCorpus":
        return cls.from_texts(iter_jsonl_text(path, text_key=text_key), tokenizer,
                              append_eos=append_eos)

    # ------------------------------------------------------------------ the .pt artifact
    def save(self, path) -> None:
        """Write the version-2 artifact; an existing file is never overwritten."""
        if self.is_legacy:
            raise ValueError("a legacy (tensor-only) corpus has no tokenizer metadata to save")
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        payload: dict[str, Any] = {"artifact": ARTIFACT_NAME, "format_version": ARTIFACT_VERSION,
                                   "fingerprint": self.fingerprint}
        payload.update({k: getattr(self, k) for k in _PAYLOAD + _META})
        try:
            f = target.open("xb")
        except FileExistsError as e:
            raise FileExistsError(f"{target} exists; token corpora are never overwritten") from e
        try:
            with f:
                torch.save(payload, f)
        except BaseException:
            target.unlink(missing_ok=True)
            raise

    @classmethod
    def load(cls, path) -> "TokenCorpus":
        obj = torch.load(Path(path), map_location="cpu", weights_only=True)
        if isinstance(obj, dict) and set(obj) == {"tokens"}:
            obj = obj["tokens"]
            if not isinstance(obj, torch.Tensor):
                raise TypeError("legacy {'tokens': ...} file does not hold a tensor")
        if isinstance(obj, torch.Tensor):
            return cls._legacy(obj)
        if not isinstance(obj, dict):
            raise TypeError(f"{path}: not a token corpus (got {type(obj).__name__})")
        if obj.get("artifact") != ARTIFACT_NAME:
            raise ValueError(f"{path}: artifact {obj.get('artifact')!r} is not a token corpus")
        version = obj.get("format_version")
        want = _KEYS_BY_VERSION.get(version) if _is_int(version) else None
        if want is None:
            raise ValueError(f"{path}: token corpus format_version {version!r} is not 1 or 2")
        missing, extra = sorted(want - set(obj)), sorted(set(obj) - want)
        if missing or extra:
            raise ValueError(f"{path}: malformed token corpus (missing keys: {missing or '-'}; "
                             f"unknown keys: {extra or '-'})")
        corpus = cls(**{k: obj[k] for k in _PAYLOAD + _META})
        if version == 2:
            stored = obj["fingerprint"]
            if not (isinstance(stored, str) and len(stored) == 64 and
                    all(c in "0123456789abcdefABCDEF" for c in stored)):
                raise ValueError(f"{path}: stored fingerprint is not a SHA-256 hex digest")
            if stored != corpus.fingerprint:
                raise ValueError(f"{path}: content fingerprint does not match the stored one "
                                 "(corrupted or edited file)")
        return corpus

    @classmethod
    def _legacy(cls, t: torch.Tensor) -> "TokenCorpus":
        t = _as_int_vector("legacy tokens", t)
        if t.numel() and int(t.min()) < 0:
            raise ValueError("legacy token ids must be >= 0")
        vocab = int(t.max()) + 1 if t.numel() else 1
        return cls(tokens=t, document_offsets=torch.tensor([0, t.numel()]), documents=1,
                   vocab_size=vocab, eos_id=None, tokenizer_fingerprint=None, append_eos=False)


def build_token_corpus(texts: Iterable[str], tokenizer, *, append_eos: bool = True
                       ) -> TokenCorpus:
    return TokenCorpus.from_texts(texts, tokenizer, append_eos=append_eos)


def preprocess_jsonl(input_path, output_path, tokenizer, *, text_key: str = "text",
                     append_eos: bool = True) -> TokenCorpus:
    """JSONL file -> saved ``.pt`` corpus (returned)."""
    corpus = TokenCorpus.from_jsonl(input_path, tokenizer, text_key=text_key,
                                    append_eos=append_eos)
    corpus.save(output_path)
    return corpus
