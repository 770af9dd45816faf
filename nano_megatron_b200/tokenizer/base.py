"""Tokenizer protocol, special tokens and training configuration.

Same contract as the reference (src/nano_megatron/tokenizer/base.py:21-157):
four control-form special tokens (``<|name|>``) in the fixed order unk, bos,
eos, pad (ids 0..3 for freshly trained artifacts).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Protocol, Sequence

CONTROL_TOKEN = re.compile(r"^<\|[A-Za-z0-9_.:-]+\|>$")


class TextTokenizer(Protocol):
    vocab_size: int
    fingerprint: str
    unk_token_id: int
    bos_token_id: int
    eos_token_id: int
    pad_token_id: int

    def encode(self, text: str, *, add_bos: bool = False, add_eos: bool = False) -> list[int]: ...

    def encode_batch(self, texts: Sequence[str], *, add_bos: bool = False,
                     add_eos: bool = False) -> list[list[int]]: ...

    def decode(self, token_ids: Sequence[int], *, skip_special_tokens: bool = True) -> str: ...


@dataclass(frozen=True, slots=True)
class SpecialTokens:
    unk: str = "<|unk|>"
    bos: str = "<|bos|>"
    eos: str = "<|endoftext|>"
    pad: str = "<|pad|>"

    def __post_init__(self) -> None:
        from tokenizers.pre_tokenizers import ByteLevel

        values = self.as_dict()
        for role, tok in values.items():
            if not isinstance(tok, str):
                raise TypeError(f"special token {role!r} must be a string")
            if tok == "":
                raise ValueError(f"special token {role!r} cannot be empty")
            if CONTROL_TOKEN.fullmatch(tok) is None:
                raise ValueError(f"special token {role!r} must use the reserved control form "
                                 "'<|name|>' with an ASCII name")
        if len(set(values.values())) != len(values):
            raise ValueError("unk, bos, eos and pad special tokens must be unique")
        alphabet = set(ByteLevel.alphabet())
        clash = [r for r, t in values.items() if t in alphabet]
        if clash:
            raise ValueError("special tokens must not overlap single-symbol byte-level alphabet "
                             "entries: " + ", ".join(clash))

    def as_dict(self) -> dict[str, str]:
        return {"unk": self.unk, "bos": self.bos, "eos": self.eos, "pad": self.pad}

    def ordered(self) -> tuple[str, str, str, str]:
        return self.unk, self.bos, self.eos, self.pad


@dataclass(frozen=True, slots=True)
class ByteBPETrainingConfig:
    vocab_size: int
    min_frequency: int = 2
    special_tokens: SpecialTokens = field(default_factory=SpecialTokens)
    show_progress: bool = False

    def __post_init__(self) -> None:
        from tokenizers.pre_tokenizers import ByteLevel

        for name in ("vocab_size", "min_frequency"):
            v = getattr(self, name)
            if isinstance(v, bool) or not isinstance(v, int):
                raise TypeError(f"{name} must be an integer")
            if v < 1:
                raise ValueError(f"{name} must be positive")
        if not isinstance(self.special_tokens, SpecialTokens):
            raise TypeError("special_tokens must be a SpecialTokens instance")
        if not isinstance(self.show_progress, bool):
            raise TypeError("show_progress must be a boolean")
        need = len(set(ByteLevel.alphabet()) | set(self.special_tokens.ordered()))
        if self.vocab_size < need:
            raise ValueError(f"vocab_size must be at least {need} to keep every byte and special "
                             "token")
