"""Model families (the dense GPT in :mod:`.gpt`)."""

from .gpt import GPTModel, GPTModelBuilder, GPTOutput

__all__ = ["GPTModel", "GPTModelBuilder", "GPTOutput"]
