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


# (head_dim, q heads, kv heads, query rows, key rows, batch, causal, q_offset, k_offset):
# square causal blocks, a non-causal block, and an off-diagonal causal block of a longer
# sequence (queries 384.. of a 640-token sequence against keys 128..), as context
# parallelism issues them
CASES = [(64, 4, 2, 256, 256, 2, 1, 0, 0), (128, 4, 4, 192, 192, 1, 1, 0, 0),
         (64, 4, 2, 128, 320, 2, 0, 0, 0), (64, 2, 1, 256, 192, 1, 1, 384, 128)]


@pytest.mark.parametrize("d,hq,hkv,sq,sk,b,causal,qo,ko", CASES)
def test_noalloc_backward_matches_regular_entry_point(d, hq, hkv, sq, sk, b, causal, qo, ko):
    from nano_megatron_b200.ops import lib

    fn, strerror = _load_symbol()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(11)
    q = torch.randn(b, sq, hq, d, device=dev).bfloat16()
    k = torch.randn(b, sk, hkv, d, device=dev).bfloat16()
    v = torch.randn(b, sk, hkv, d, device=dev).bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(b, hq, sq, device=dev)
    scale = 1.0 / math.sqrt(d)
    lib().flash_attn_fwd(q, k, v, o, lse, scale, bool(causal), qo, ko)
    do = torch.randn_like(o)
    # regular entry point (workspaces allocated by the caller)
    dq_ref, dk_ref, dv_ref = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(b * hq * sq, device=dev)
    dq_acc = torch.empty(b * sq * hq * d, device=dev)
    lib().flash_attn_bwd(q, k, v, o, do, lse, dq_ref, dk_ref, dv_ref, delta, dq_acc, scale,
                         bool(causal), qo, ko, None, None, None)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row share (and must re-clear) the scratch
        dq, dk, dv = torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0)
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, sq, sk, hq, hkv,
                d, scale, causal, qo, ko, stream)
        torch.cuda.synchronize()
        assert rc == 0, strerror(rc).decode()
        assert _rel(dq, dq_ref) < 1e-2
        assert _rel(dk, dk_ref) < 1e-2
        assert _rel(dv, dv_ref) < 1e-2


def _attention_fp32(q, k, v, scale, causal, qo, ko):
    """Plain fp32 PyTorch attention with GQA (k/v heads repeated) and absolute offsets."""
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))     # [B, H, S, D]
    rep = qf.shape[1] // kf.shape[1]
    kf, vf = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        qi = torch.arange(q.shape[1], device=q.device)[:, None] + qo
        ki = torch.arange(k.shape[1], device=q.device)[None, :] + ko
        s = s.masked_fill(ki > qi, float("-inf"))
    return (s.softmax(-1) @ vf).transpose(1, 2)


def test_noalloc_backward_matches_fp32_autograd():
    """Against an fp32 PyTorch autograd reference of the same attention (not only the
    regular entry point, which runs the same kernels)."""
    from nano_megatron_b200.ops import lib

    fn, strerror = _load_symbol()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(5)
    b, sq, sk, hq, hkv, d, qo, ko = 1, 128, 192, 4, 2, 64, 64, 0
    q = torch.randn(b, sq, hq, d, device=dev).bfloat16()
    k = torch.randn(b, sk, hkv, d, device=dev).bfloat16()
    v = torch.randn(b, sk, hkv, d, device=dev).bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(b, hq, sq, device=dev)
    scale = 1.0 / math.sqrt(d)
    lib().flash_attn_fwd(q, k, v, o, lse, scale, True, qo, ko)
    do = torch.randn_like(o)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref = _attention_fp32(qr, kr, vr, scale, True, qo, ko)
    ref.backward(do.float())
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
            lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, sq, sk, hq, hkv, d,
            scale, 1, qo, ko, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, strerror(rc).decode()
    assert _rel(dq, qr.grad) < 2e-2
    assert _rel(dk, kr.grad) < 2e-2
    assert _rel(dv, vr.grad) < 2e-2


def test_noalloc_without_keys_writes_zero_dq():
    fn, strerror = _load_symbol()
    dev = torch.device("cuda", torch.cuda.current_device())
    b, sq, hq, d = 1, 64, 2, 64
    q = torch.randn(b, sq, hq, d, device=dev).bfloat16()
    kv = torch.zeros(16, device=dev, dtype=torch.bfloat16)     # no keys: never read
    o = torch.randn_like(q)
    do = torch.randn_like(q)
    lse = torch.zeros(b, hq, sq, device=dev)
    dq = torch.full_like(q, 7.0)
    rc = fn(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), o.data_ptr(), do.data_ptr(),
            lse.data_ptr(), dq.data_ptr(), kv.data_ptr(), kv.data_ptr(), b, sq, 0, hq, hq, d,
            0.125, 1, 0, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, strerror(rc).decode()
    assert torch.count_nonzero(dq) == 0


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
