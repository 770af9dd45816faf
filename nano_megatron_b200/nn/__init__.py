"""Model building blocks: norms, rotary embedding, dropout, activation checkpointing, and
the kernel backend (:mod:`.kernels`)."""

from .activation_checkpoint import ActivationCheckpoint, activation_checkpoint
from .dropout import activation_rng_context, make_dropout, parallel_dropout
from .kernels import B200KernelBackend, KernelBackend, build_kernel_backend
from .norms import RMSNorm
from .rotary import RotaryEmbedding, apply_rotary_pos_emb, rope_inv_freq, rotate_half

__all__ = [n for n in dir() if not n.startswith("_")]
