"""Fixed-length causal-LM datasets: sample ``i`` is the window ``tokens[i*S : i*S+S+1]``.

Windows overlap by one token (stride ``S``), giving ``(N - 1) // S`` samples;
``input_ids``/``labels`` are the window without its last/first token. Each
dataset exposes a fingerprint (sha256 of a canonical JSON record naming the
algorithm, the corpus fingerprint and ``S``) and, for token-stream datasets, a
native window source so the loader can gather whole batches in C++. Sample
definitions, fingerprints and the random-token generator (``torch.Generator``
seeded ``seed + index``) follow the reference
(src/nano_megatron/data/datasets.py:93-369) so the same config yields the
same samples in both frameworks.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch
from torch.utils.data import Dataset

from .corpus import TokenCorpus
from .mmap_corpus import MMapTokenCorpus

_INT_DTYPES = (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64)


def _sha_json(obj) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, separators=(",", ":"))
                          .encode("utf-8")).hexdigest()


def fixed_length_fingerprint(corpus_fp: str, seq: int) -> str:
    if not isinstance(corpus_fp, str) or not corpus_fp:
        raise ValueError("corpus_fingerprint must be a non-empty string")
    return _sha_json({"algorithm": "fixed-length-causal-v1", "corpus": corpus_fp,
                      "sequence_length": seq})


def _check_seq(seq) -> int:
    if isinstance(seq, bool) or not isinstance(seq, int) or seq < 1:
        raise ValueError("sequence_length must be positive")
    return seq


class _WindowDataset(Dataset):
    sequence_length: int
    num_samples: int

    def __len__(self) -> int:
        return self.num_samples

    @property
    def window_size(self) -> int:
        return self.sequence_length + 1

    def window_starts(self, indices: torch.Tensor) -> torch.Tensor:
        return indices.to(torch.int64) * self.sequence_length

    def _check(self, index: int) -> None:
        if not 0 <= index < self.num_samples:
            raise IndexError(index)

    def __getitem__(self, index: int) -> dict[str, torch.Tensor]:
        self._check(index)
        out = torch.empty(1, self.window_size, dtype=torch.int64)
        self.native_source().gather(self.window_starts(torch.tensor([index])), self.window_size,
                                    out, 1)
        w = out[0]
        return {"input_ids": w[:-1], "labels": w[1:]}


class FixedLengthTokenDataset(_WindowDataset):
    def __init__(self, tokens: torch.Tensor, sequence_length: int, *,
                 corpus_fingerprint: str | None = None) -> None:
        if not isinstance(tokens, torch.Tensor):
            raise TypeError("tokens must be a torch.Tensor")
        if tokens.ndim != 1:
            raise ValueError("tokens must be a one-dimensional tensor")
        if tokens.dtype not in _INT_DTYPES:
            raise TypeError("tokens must use an integer dtype")
        self.tokens = tokens.to(dtype=torch.long, device="cpu").contiguous()
        self.sequence_length = _check_seq(sequence_length)
        self.num_samples = max(0, (self.tokens.numel() - 1) // self.sequence_length)
        if self.num_samples < 1:
            raise ValueError("token tensor is too short for one training sample")
        if corpus_fingerprint is None:
            h = hashlib.sha256(b"nano-megatron-flat-token-stream-v1\0")
            h.update(self.tokens.numpy().astype("<i8", copy=False).tobytes(order="C"))
            corpus_fingerprint = h.hexdigest()
        self.fingerprint = fixed_length_fingerprint(corpus_fingerprint, self.sequence_length)
        self._src = None

    @classmethod
    def from_file(cls, path, sequence_length: int) -> "FixedLengthTokenDataset":
        c = TokenCorpus.load(path)
        return cls(c.tokens, sequence_length, corpus_fingerprint=c.fingerprint)

    def native_source(self):
        if self._src is None:
            from nano_megatron_b200.native import native

            self._src = native().TokenSource(self.tokens)
        return self._src

    def __getstate__(self):
        s = dict(self.__dict__)
        s["_src"] = None
        return s


class MMapTokenDataset(_WindowDataset):
    """Windows read straight from an mmap corpus; nothing is materialised."""

    def __init__(self, artifact_dir, sequence_length: int) -> None:
        self.sequence_length = _check_seq(sequence_length)
        c = MMapTokenCorpus.load(artifact_dir)
        self.artifact_dir = Path(c.path)
        self.token_count = int(c.token_count)
        self.document_count = self.documents = int(c.documents)
        self.vocab_size = int(c.vocab_size)
        self.eos_id = int(c.eos_id)
        self.tokenizer_fingerprint = str(c.tokenizer_fingerprint)
        self.append_eos = bool(c.append_eos)
        self.corpus_fingerprint = str(c.fingerprint)
        self.num_samples = max(0, (self.token_count - 1) // self.sequence_length)
        if self.num_samples < 1:
            raise ValueError("mmap token corpus is too short for one training sample")
        self.fingerprint = fixed_length_fingerprint(self.corpus_fingerprint,
                                                    self.sequence_length)
        self._corpus = c

    def native_source(self):
        return self._corpus.native_source()

    def read_window_numpy(self, index: int) -> np.ndarray:
        self._check(index)
        s = index * self.sequence_length
        return np.array(self._corpus.read_tokens(s, s + self.window_size), dtype=np.int64)

    def __getstate__(self):
        return dict(self.__dict__)


class RandomTokenDataset(Dataset):
    """Deterministic synthetic tokens: sample ``i`` draws from a generator seeded ``seed + i``."""

    def __init__(self, *, num_samples: int, sequence_length: int, vocab_size: int,
                 seed: int = 1234) -> None:
        if min(num_samples, sequence_length, vocab_size) < 1:
            raise ValueError("dataset sizes must be positive")
        self.num_samples, self.sequence_length = num_samples, sequence_length
        self.vocab_size, self.seed = vocab_size, seed
        self.fingerprint = _sha_json({"algorithm": "random-token-dataset-v1",
                                      "num_samples": num_samples, "seed": seed,
                                      "sequence_length": sequence_length,
                                      "vocab_size": vocab_size})

    def __len__(self) -> int:
        return self.num_samples

    def window(self, index: int) -> torch.Tensor:
        if not 0 <= index < self.num_samples:
            raise IndexError(index)
        g = torch.Generator().manual_seed(self.seed + index)
        return torch.randint(self.vocab_size, (self.sequence_length + 1,), generator=g)

    def __getitem__(self, index: int) -> dict[str, torch.Tensor]:
        w = self.window(index)
        return {"input_ids": w[:-1], "labels": w[1:]}


def _append_eos(data) -> bool:
    tc = getattr(data, "tokenizer", None)
    if tc is None:
        raise ValueError("data.text_path requires data.tokenizer configuration")
    if not isinstance(tc.append_eos, bool):
        raise TypeError("data.tokenizer.append_eos must be a boolean")
    return tc.append_eos


def _same_vocab(actual: int, expected: int, source: str) -> None:
    if actual != expected:
        raise ValueError(f"{source} vocab_size ({actual}) does not match model.vocab_size "
                         f"({expected})")


def _check_structured(c, *, vocab: int, tokenizer, append: bool | None, source: str) -> None:
    _same_vocab(c.vocab_size, vocab, source)
    if tokenizer is not None:
        _same_vocab(tokenizer.vocab_size, vocab, "tokenizer")
        if tokenizer.eos_token_id != c.eos_id:
            raise ValueError("tokenizer.eos_token_id does not match token corpus eos_id")
        if tokenizer.fingerprint != c.tokenizer_fingerprint:
            raise ValueError("tokenizer fingerprint does not match token corpus metadata")
    if append is not None and c.append_eos != append:
        raise ValueError("token corpus append_eos does not match data.tokenizer.append_eos")


def build_train_dataset(config, tokenizer=None, *, data_config=None):
    """Random, pre-tokenised (``.pt`` or mmap) or JSONL data, per the config."""
    seq, vocab = int(config.model.seq_length), int(config.model.vocab_size)
    data = config.data if data_config is None else data_config
    text, pt, mm = (getattr(data, n, None) for n in ("text_path", "path", "mmap_path"))
    if sum(p is not None for p in (text, pt, mm)) > 1:
        raise ValueError("data.path, data.mmap_path and data.text_path are mutually exclusive")
    if text is not None:
        if tokenizer is None:
            raise ValueError("data.text_path requires an explicitly supplied tokenizer")
        _same_vocab(tokenizer.vocab_size, vocab, "tokenizer")
        c = TokenCorpus.from_jsonl(text, tokenizer, text_key=data.text_key,
                                   append_eos=_append_eos(data))
        return FixedLengthTokenDataset(c.tokens, seq, corpus_fingerprint=c.fingerprint)
    tc = getattr(data, "tokenizer", None)
    if (mm is not None or pt is not None) and tc is not None and tokenizer is None:
        raise ValueError("data.tokenizer configuration requires an explicitly supplied "
                         "tokenizer")
    append = None if tc is None else _append_eos(data)
    if mm is not None:
        ds = MMapTokenDataset(mm, seq)
        _check_structured(ds, vocab=vocab, tokenizer=tokenizer, append=append,
                          source="mmap token corpus")
        return ds
    if pt is not None:
        c = TokenCorpus.load(pt)
        if c.is_legacy:
            if tokenizer is not None:
                _same_vocab(tokenizer.vocab_size, vocab, "tokenizer")
            if c.tokens.numel() and int(c.tokens.max()) >= vocab:
                raise ValueError("legacy token file contains ids outside model.vocab_size")
            if append is not None:
                raise ValueError("legacy token files do not record append_eos; omit "
                                 "data.tokenizer or preprocess into a structured TokenCorpus")
        else:
            _check_structured(c, vocab=vocab, tokenizer=tokenizer, append=append,
                              source="token corpus")
        return FixedLengthTokenDataset(c.tokens, seq, corpus_fingerprint=c.fingerprint)
    local = int(config.training.micro_batch_size) * int(config.training.gradient_accumulation_steps)
    replicas = int(getattr(config.parallel, "data", None) or 1) * int(config.parallel.expert)
    return RandomTokenDataset(num_samples=max(int(config.training.max_steps) * local * replicas,
                                              1024),
                              sequence_length=seq, vocab_size=vocab,
                              seed=int(config.training.seed))
