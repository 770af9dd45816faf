"""Byte-level BPE tokenizer on the HuggingFace ``tokenizers`` library.

Artifact directory = ``tokenizer.json`` (backend) + ``metadata.json`` (format
``nano-megatron-byte-level-bpe`` v1, vocab size, special tokens and ids,
fingerprint = sha256 of the canonical backend JSON). Special-looking text in
documents stays text (``encode_special_tokens``); BOS/EOS are only added by the
explicit flags. Same artifact format as the reference
(src/nano_megatron/tokenizer/byte_bpe.py:110-505), so artifacts are
interchangeable.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from collections.abc import Iterable, Iterator, Sequence
from pathlib import Path
from typing import Any

from .base import ByteBPETrainingConfig, SpecialTokens

ARTIFACT_FORMAT = "nano-megatron-byte-level-bpe"
ARTIFACT_VERSION = 1
TOKENIZER_FILE = "tokenizer.json"
METADATA_FILE = "metadata.json"
ROLES = ("unk", "bos", "eos", "pad")


class TokenizerArtifactError(ValueError):
    pass


def _backend_json(backend) -> dict[str, Any]:
    try:
        payload = json.loads(backend.to_str())
    except (TypeError, ValueError) as error:
        raise TokenizerArtifactError("tokenizer backend did not produce valid JSON") from error
    if not isinstance(payload, dict):
        raise TokenizerArtifactError("tokenizer backend JSON must contain an object")
    return payload


def _fingerprint(backend) -> str:
    canon = json.dumps(_backend_json(backend), ensure_ascii=False, sort_keys=True,
                       separators=(",", ":")).encode("utf-8")
    return hashlib.sha256(canon).hexdigest()


def _checked_texts(texts: Iterable[str]) -> Iterator[str]:
    for i, t in enumerate(texts):
        if not isinstance(t, str):
            raise TypeError(f"training text {i} must be a string, got {type(t).__name__}")
        yield t


class ByteLevelBPETokenizer:
    def __init__(self, backend, special_tokens: SpecialTokens) -> None:
        self._backend = backend
        self._backend.encode_special_tokens = True
        self._special = special_tokens
        model = _backend_json(backend).get("model", {})
        if model.get("type") != "BPE":
            raise TokenizerArtifactError("tokenizer backend must be a BPE model")
        if model.get("unk_token") != special_tokens.unk:
            raise TokenizerArtifactError("tokenizer backend unk token does not match metadata")
        ids = {}
        for role, tok in special_tokens.as_dict().items():
            tid = backend.token_to_id(tok)
            if tid is None:
                raise TokenizerArtifactError(f"tokenizer vocabulary is missing the {role!r} "
                                             f"special token {tok!r}")
            ids[role] = int(tid)
        if len(set(ids.values())) != len(ids):
            raise TokenizerArtifactError("special tokens must map to unique token ids")
        self._ids = ids
        specials = set(ids.values())
        for role, tok in special_tokens.as_dict().items():
            if specials & set(backend.encode(tok, add_special_tokens=False).ids):
                raise TokenizerArtifactError(f"{role} special token {tok!r} collides with "
                                             "ordinary text encoding")
        self._fp = _fingerprint(backend)

    # ------------------------------------------------------------------ build
    @classmethod
    def train(cls, texts: Iterable[str], config: ByteBPETrainingConfig
              ) -> "ByteLevelBPETokenizer":
        from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

        if not isinstance(config, ByteBPETrainingConfig):
            raise TypeError("config must be a ByteBPETrainingConfig instance")
        backend = Tokenizer(models.BPE(unk_token=config.special_tokens.unk))
        backend.encode_special_tokens = True
        backend.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
        backend.decoder = decoders.ByteLevel()
        trainer = trainers.BpeTrainer(vocab_size=config.vocab_size,
                                      min_frequency=config.min_frequency,
                                      show_progress=config.show_progress,
                                      special_tokens=list(config.special_tokens.ordered()),
                                      initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
        try:
            backend.train_from_iterator(_checked_texts(texts), trainer=trainer)
        except (TypeError, ValueError):
            raise
        except Exception as error:  # noqa: BLE001
            raise RuntimeError(f"byte-level BPE training failed: {error}") from error
        return cls(backend, config.special_tokens)

    @classmethod
    def load(cls, artifact_dir: str | Path) -> "ByteLevelBPETokenizer":
        from tokenizers import Tokenizer

        d = Path(artifact_dir)
        tok_path, meta_path = d / TOKENIZER_FILE, d / METADATA_FILE
        if not tok_path.is_file() or not meta_path.is_file():
            raise TokenizerArtifactError(f"tokenizer artifact is incomplete: {d}")
        try:
            meta = json.loads(meta_path.read_text(encoding="utf-8"))
        except (OSError, ValueError) as error:
            raise TokenizerArtifactError(f"could not read tokenizer metadata: {error}") from error
        if meta.get("format") != ARTIFACT_FORMAT:
            raise TokenizerArtifactError(f"unsupported tokenizer artifact format: "
                                         f"{meta.get('format')!r}")
        if meta.get("version") != ARTIFACT_VERSION:
            raise TokenizerArtifactError(f"unsupported tokenizer artifact version: "
                                         f"{meta.get('version')!r}")
        specials = meta.get("special_tokens")
        ids = meta.get("special_token_ids")
        for name, v in (("special_tokens", specials), ("special_token_ids", ids)):
            if not isinstance(v, dict) or set(v) != set(ROLES):
                raise TokenizerArtifactError(f"metadata field {name!r} must contain exactly "
                                             + ", ".join(ROLES))
        tok = cls(Tokenizer.from_file(str(tok_path)), SpecialTokens(**specials))
        if tok._ids != {k: int(v) for k, v in ids.items()}:
            raise TokenizerArtifactError("tokenizer special-token ids do not match metadata")
        if meta.get("vocab_size") != tok.vocab_size:
            raise TokenizerArtifactError("tokenizer vocab size does not match metadata")
        if meta.get("fingerprint") != tok.fingerprint:
            raise TokenizerArtifactError("tokenizer fingerprint does not match metadata")
        return tok

    def _metadata(self) -> dict[str, Any]:
        return {"format": ARTIFACT_FORMAT, "version": ARTIFACT_VERSION,
                "encode_special_tokens_as_text": True, "vocab_size": self.vocab_size,
                "special_tokens": self._special.as_dict(), "special_token_ids": dict(self._ids),
                "fingerprint": self.fingerprint}

    @staticmethod
    def validate_save_target(artifact_dir: str | Path) -> None:
        d = Path(artifact_dir)
        if d.exists() and (not d.is_dir() or any(d.iterdir())):
            raise FileExistsError(f"tokenizer artifact path already exists: {d}")

    def save(self, artifact_dir: str | Path) -> None:
        d = Path(artifact_dir)
        self.validate_save_target(d)
        d.parent.mkdir(parents=True, exist_ok=True)
        was_empty = d.is_dir()
        tmp = Path(tempfile.mkdtemp(prefix=f".{d.name}.tmp-", dir=d.parent))
        try:
            self._backend.save(str(tmp / TOKENIZER_FILE), pretty=True)
            (tmp / METADATA_FILE).write_text(json.dumps(self._metadata(), ensure_ascii=False,
                                                        indent=2, sort_keys=True) + "\n",
                                             encoding="utf-8")
            if type(self).load(tmp).fingerprint != self.fingerprint:
                raise TokenizerArtifactError("saved tokenizer fingerprint changed during "
                                             "artifact validation")
            if was_empty:
                d.rmdir()
            os.replace(tmp, d)
        finally:
            if tmp.exists():
                shutil.rmtree(tmp)

    # ------------------------------------------------------------------ use
    special_tokens = property(lambda self: self._special)
    vocab_size = property(lambda self: int(self._backend.get_vocab_size(with_added_tokens=True)))
    fingerprint = property(lambda self: self._fp)
    unk_token_id = property(lambda self: self._ids["unk"])
    bos_token_id = property(lambda self: self._ids["bos"])
    eos_token_id = property(lambda self: self._ids["eos"])
    pad_token_id = property(lambda self: self._ids["pad"])

    def _wrap(self, ids: list[int], add_bos: bool, add_eos: bool) -> list[int]:
        for name, v in (("add_bos", add_bos), ("add_eos", add_eos)):
            if not isinstance(v, bool):
                raise TypeError(f"{name} must be a boolean")
        return ([self.bos_token_id] if add_bos else []) + ids + \
            ([self.eos_token_id] if add_eos else [])

    def encode(self, text: str, *, add_bos: bool = False, add_eos: bool = False) -> list[int]:
        if not isinstance(text, str):
            raise TypeError("text must be a string")
        return self._wrap(list(self._backend.encode(text, add_special_tokens=False).ids),
                          add_bos, add_eos)

    def encode_batch(self, texts: Sequence[str], *, add_bos: bool = False,
                     add_eos: bool = False) -> list[list[int]]:
        texts = list(texts)
        if any(not isinstance(t, str) for t in texts):
            raise TypeError("texts must be strings")
        encs = self._backend.encode_batch(texts, add_special_tokens=False)
        return [self._wrap(list(e.ids), add_bos, add_eos) for e in encs]

    def decode(self, token_ids: Sequence[int], *, skip_special_tokens: bool = True) -> str:
        if not isinstance(skip_special_tokens, bool):
            raise TypeError("skip_special_tokens must be a boolean")
        ids = [int(t) for t in token_ids]
        bad = [t for t in ids if not 0 <= t < self.vocab_size]
        if bad:
            raise ValueError(f"token ids outside the vocabulary: {bad[:5]}")
        return self._backend.decode(ids, skip_special_tokens=skip_special_tokens)

    def token_to_id(self, token: str) -> int | None:
        return self._backend.token_to_id(token)

    def id_to_token(self, token_id: int) -> str | None:
        return self._backend.id_to_token(int(token_id))
