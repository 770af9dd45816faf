"""What the training stack needs from a tokenizer, and the byte-BPE training settings.

The model only sees integer ids, so a tokenizer is anything with the small interface of
:class:`TextTokenizer` (no torch involved; usable in plain preprocessing scripts).

Special tokens have four roles: unknown, begin-of-sequence, end-of-text and padding. Their
text must look like a control token, ``<|name|>`` with an ASCII name, so it can never be
produced by ordinary text through the byte-level alphabet; they are handed to the BPE
trainer in the order unk, bos, eos, pad, which gives them ids 0..3 in a freshly trained
vocabulary. The default strings, that order and the control form are the reference's
(src/nano_megatron/tokenizer/base.py), so artifacts trained by either framework load in
the other.
"""

from __future__ import annotations

import re
from dataclasses import astuple, dataclass, field, fields
from typing import Protocol, Sequence

CONTROL_TOKEN = re.compile(r"^<\|[A-Za-z0-9_.:-]+\|>$")


def _byte_alphabet() -> set[str]:
    from tokenizers.pre_tokenizers import ByteLevel

    return set(ByteLevel.alphabet())


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
        roles = self.as_dict()
        for role, text in roles.items():
            if not isinstance(text, str):
                raise TypeError(f"{role} token is a {type(text).__name__}, not text")
            if not CONTROL_TOKEN.fullmatch(text):
                raise ValueError(f"{role} token {text!r} is not of the form '<|name|>' "
                                 "(name: letters, digits, '_', '.', ':', '-')")
        seen: dict[str, str] = {}
        for role, text in roles.items():
            if text in seen:
                raise ValueError(f"{role} and {seen[text]} tokens are both {text!r}")
            seen[text] = role
        in_alphabet = sorted(r for r, t in roles.items() if t in _byte_alphabet())
        if in_alphabet:
            raise ValueError("special tokens collide with byte-level alphabet symbols: " +
                             ", ".join(in_alphabet))

    def as_dict(self) -> dict[str, str]:
        """role -> text, in id order (unk, bos, eos, pad)."""
        return {f.name: getattr(self, f.name) for f in fields(self)}

    def ordered(self) -> tuple[str, str, str, str]:
        """The texts in the order the BPE trainer receives them (ids 0..3)."""
        return astuple(self)


def _count_field(name: str, value) -> None:
    if type(value) is not int:
        raise TypeError(f"{name} must be an int, got {value!r}")
    if value <= 0:
        raise ValueError(f"{name} must be >= 1, got {value}")


@dataclass(frozen=True, slots=True)
class ByteBPETrainingConfig:
    vocab_size: int
    min_frequency: int = 2
    special_tokens: SpecialTokens = field(default_factory=SpecialTokens)
    show_progress: bool = False

    def __post_init__(self) -> None:
        _count_field("vocab_size", self.vocab_size)
        _count_field("min_frequency", self.min_frequency)
        if not isinstance(self.special_tokens, SpecialTokens):
            raise TypeError(f"special_tokens is a {type(self.special_tokens).__name__}, "
                            "expected SpecialTokens")
        if type(self.show_progress) is not bool:
            raise TypeError(f"show_progress must be a bool, got {self.show_progress!r}")
        # every one of the 256 byte symbols stays in the vocabulary (unseen bytes must
        # still encode), plus the special tokens
        floor = len(_byte_alphabet() | set(self.special_tokens.ordered()))
        if self.vocab_size < floor:
            raise ValueError(f"vocab_size={self.vocab_size} cannot hold the byte alphabet and "
                             f"the special tokens ({floor} entries)")
