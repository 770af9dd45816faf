"""Command-line entry points: train, export, generate, tokenizer, tinystories."""
