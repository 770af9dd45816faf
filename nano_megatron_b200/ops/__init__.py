"""Kernel entry points (sm_100a CUDA) and their PyTorch reference formulas."""

from ._ext import available, check_status, lib, status_word

__all__ = ["available", "check_status", "lib", "status_word"]
