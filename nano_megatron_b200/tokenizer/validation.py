"""Tokenizer/model compatibility: ids must fit the model's unpadded vocabulary exactly."""

from __future__ import annotations


def validate_tokenizer_for_model(tokenizer, model_config) -> None:
    tv, mv = int(tokenizer.vocab_size), int(model_config.vocab_size)
    if tv != mv:
        raise ValueError("tokenizer and model vocabulary sizes must match exactly: "
                         f"tokenizer.vocab_size={tv}, model_config.vocab_size={mv}")
    ids = {}
    for name in ("unk_token_id", "bos_token_id", "eos_token_id", "pad_token_id"):
        tid = getattr(tokenizer, name)
        if isinstance(tid, bool) or not isinstance(tid, int):
            raise TypeError(f"tokenizer.{name} must be an integer, got {tid!r}")
        if not 0 <= tid < tv:
            raise ValueError(f"tokenizer.{name}={tid} is outside vocabulary range [0, {tv})")
        ids[name] = tid
    if len(set(ids.values())) != len(ids):
        raise ValueError(f"tokenizer special-token ids must be unique: {ids}")
