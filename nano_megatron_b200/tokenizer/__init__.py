"""Byte-level BPE tokenizer (artifact-compatible with the reference)."""

from .base import ByteBPETrainingConfig, SpecialTokens, TextTokenizer
from .byte_bpe import ByteLevelBPETokenizer, TokenizerArtifactError
from .validation import validate_tokenizer_for_model

__all__ = ["ByteBPETrainingConfig", "ByteLevelBPETokenizer", "SpecialTokens", "TextTokenizer",
           "TokenizerArtifactError", "validate_tokenizer_for_model"]
