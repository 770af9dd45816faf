"""Loader for the host-only native runtime extension (``_native``: data loading)."""

from __future__ import annotations

import functools
import importlib


@functools.lru_cache(maxsize=1)
def native():
    try:
        return importlib.import_module("nano_megatron_b200._native")
    except ImportError as e:
        raise ImportError("the nano_megatron_b200._native extension is not built; run "
                          "`python setup.py build_ext --inplace`") from e
