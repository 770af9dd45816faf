"""Loader for the in-tree sm_100a kernel library ``nano_megatron_b200._C``.

On a CUDA device every op in :mod:`nano_megatron_b200.ops` runs through this
library; if it cannot be imported the op raises instead of silently running a
PyTorch substitute. The pure-PyTorch formulas in :mod:`.reference` exist only
for CPU tensors (the gloo test suite and CPU smoke runs) and as test oracles.
"""

from __future__ import annotations

import functools

import torch

_IMPORT_ERROR: Exception | None = None
try:  # pragma: no cover - depends on the build
    from nano_megatron_b200 import _C as _lib
except Exception as error:  # noqa: BLE001
    _lib = None
    _IMPORT_ERROR = error


def available() -> bool:
    return _lib is not None


def lib():
    """Return the compiled module or raise loudly."""
    if _lib is None:
        raise RuntimeError(
            "nano_megatron_b200._C (the sm_100a kernel library) is not built or failed to load: "
            f"{_IMPORT_ERROR!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return _lib


@functools.lru_cache(maxsize=None)
def _status_word(device_index: int) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", device_index))


def status_word(device: torch.device) -> torch.Tensor:
    """Device status word written by bounded waits that ran out (0 = healthy)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    return _status_word(index)


STATUS_NAMES = {
    0x101: "GEMM producer wait timed out",
    0x102: "GEMM MMA wait timed out",
    0x103: "GEMM epilogue wait timed out",
    0x201: "attention wait timed out",
    0x301: "peer flag wait timed out",
    0x302: "peer barrier wait timed out",
    0x401: "data-parallel replica flag wait timed out",
    0x501: "context-parallel flag wait timed out",
}


def check_status(device: torch.device) -> None:
    """Raise if any kernel on ``device`` reported a timed-out wait (host sync)."""
    code = int(status_word(device).item())
    if code != 0:
        raise RuntimeError(
            f"device kernel reported status 0x{code:x}: {STATUS_NAMES.get(code, 'unknown')}"
        )
