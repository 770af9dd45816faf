"""GPU test of the allocation-free flash-attention backward (``nmb_flash_attn_bwd_noalloc``).

That entry point serves callers that may not allocate device memory (code
inside an allocator's callbacks, runtimes that reserved all memory up front,
non-PyTorch hosts that own every buffer): its two temporaries come from a fixed
array inside the library. This test calls it through its exported C symbol
(ctypes, no PyTorch binding) twice in a row and checks both results against the
regular ``flash_attn_bwd`` entry point, which takes caller-allocated workspaces.
The file name sorts last so that a run stopping at the first failure has run
every other test first.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _load_symbol():
    import nano_megatron_b200._C as ext

    so = ctypes.CDLL(ext.__file__)
    fn = so.nmb_flash_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int] * 6 + [ctypes.c_float] + \
        [ctypes.c_int] * 3 + [ctypes.c_void_p]
    err = so.nmb_noalloc_strerror
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


@pytest.mark.parametrize("d,hq,hkv,s,b", [(64, 4, 2, 256, 2), (128, 4, 4, 192, 1)])
def test_noalloc_backward_matches_regular_entry_point(d, hq, hkv, s, b):
    from nano_megatron_b200.ops import lib

    fn, strerror = _load_symbol()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(11)
    q = torch.randn(b, s, hq, d, device=dev).bfloat16()
    k = torch.randn(b, s, hkv, d, device=dev).bfloat16()
    v = torch.randn(b, s, hkv, d, device=dev).bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(b, hq, s, device=dev)
    scale = 1.0 / math.sqrt(d)
    lib().flash_attn_fwd(q, k, v, o, lse, scale, True, 0, 0)
    do = torch.randn_like(o)
    # regular entry point (workspaces allocated by the caller)
    dq_ref, dk_ref, dv_ref = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(b * hq * s, device=dev)
    dq_acc = torch.empty(b * s * hq * d, device=dev)
    lib().flash_attn_bwd(q, k, v, o, do, lse, dq_ref, dk_ref, dv_ref, delta, dq_acc, scale,
                         True, 0, 0, None, None, None)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row share (and must re-clear) the scratch
        dq, dk, dv = torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0)
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, s, s, hq, hkv, d,
                scale, 1, 0, 0, stream)
        torch.cuda.synchronize()
        assert rc == 0, strerror(rc).decode()
        assert _rel(dq, dq_ref) < 1e-2
        assert _rel(dk, dk_ref) < 1e-2
        assert _rel(dv, dv_ref) < 1e-2


def test_noalloc_rejects_oversized_problem():
    fn, strerror = _load_symbol()
    dev = torch.device("cuda", torch.cuda.current_device())
    t = torch.zeros(16, device=dev, dtype=torch.bfloat16)
    lse = torch.zeros(16, device=dev)
    p = t.data_ptr()
    # B*Hq*Sq*(D+1) = 1 * 64 * 4096 * 129 floats > 8 Mi floats
    rc = fn(p, p, p, p, p, lse.data_ptr(), p, p, p, 1, 4096, 4096, 64, 64, 128, 0.1, 1, 0, 0,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert "too large" in strerror(rc).decode()
