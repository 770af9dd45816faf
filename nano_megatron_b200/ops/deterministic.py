"""Deterministic kernel mode.

By default several backward kernels sum fp32 partials with atomics, in an order the
hardware schedule decides: split-K weight gradients, the attention backward's dQ (one
partial per key block), the RMSNorm weight gradient and the embedding backward (one
partial per token). Two runs of the same step then agree to fp32 rounding but not bit for
bit. With the mode on, each of those sums runs in a fixed order instead:

* weight-gradient GEMMs run without split-K (one writer per output tile);
* the attention backward stores each key block's dQ partial into its own zeroed slot and
  ``slots_sum`` adds the slots in key-block order;
* the RMSNorm weight gradient is summed per row chunk, then the chunks in order;
* the embedding backward sorts the tokens by id (stable) and one warp adds each run of
  equal ids in token order, also on the fused tensor-parallel path.

Everything else on the training path already reduces in a fixed order (the forward, the
cross-entropy, the fused TP/DP/CP collectives, the grad norm, AdamW), so with the mode on
a step is bitwise reproducible for a fixed configuration and world size. It costs speed:
the unsplit weight-gradient GEMMs fill fewer SMs and the extra passes re-read their
inputs. CPU formulas are deterministic either way.

The switch is process-wide (the kernel library holds one flag). It is set from
``kernels.deterministic`` when the training components are built, from the environment
variable ``NMB_DETERMINISTIC=1`` at import, or with :func:`set_deterministic` /
:func:`deterministic`.
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Iterator

from . import _ext

_enabled = False


def set_deterministic(enabled: bool) -> None:
    """Turn the deterministic kernel mode on or off for this process."""
    global _enabled
    _enabled = bool(enabled)
    if _ext.available():
        _ext.lib().set_deterministic(_enabled)


def is_deterministic() -> bool:
    return _enabled


@contextlib.contextmanager
def deterministic(enabled: bool = True) -> Iterator[None]:
    """Run the enclosed block with the mode set to ``enabled``, then restore it."""
    before = _enabled
    set_deterministic(enabled)
    try:
        yield
    finally:
        set_deterministic(before)


def _env_default() -> bool:
    return os.environ.get("NMB_DETERMINISTIC", "0") not in ("", "0")


def configure(from_config: bool) -> None:
    """Apply ``kernels.deterministic`` (on if the config or the environment asks)."""
    set_deterministic(bool(from_config) or _env_default())


if _env_default():
    set_deterministic(True)
