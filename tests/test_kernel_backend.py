"""The kernel-backend seam (``nn.kernels``): linear, RMSNorm and local attention against
plain PyTorch (CPU here; the same calls on a B200 in ``test_zzz_kernel_backend_gpu.py``)."""

import math

import pytest
import torch

from nano_megatron_b200.config import config_from_dict
from nano_megatron_b200.nn.kernels import TorchKernelBackend, build_kernel_backend


def test_backend_is_selected_by_either_spelling():
    for name in ("b200", "torch"):
        kb = build_kernel_backend(config_from_dict({"kernels": {"backend": name}}).kernels)
        assert kb.name == "b200"
    assert TorchKernelBackend is type(kb)
    with pytest.raises(ValueError):
        build_kernel_backend("triton")


def test_linear_matches_nn_linear_forward_and_backward():
    torch.manual_seed(0)
    kb = build_kernel_backend("b200")
    lin = kb.linear(24, 16, bias=True)
    ref = torch.nn.Linear(24, 16)
    ref.load_state_dict(lin.state_dict())
    x = torch.randn(3, 5, 24, requires_grad=True)
    xr = x.detach().clone().requires_grad_()
    y, yr = lin(x), ref(xr)
    assert torch.allclose(y, yr, atol=1e-5)
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g)
    assert torch.allclose(x.grad, xr.grad, atol=1e-5)
    assert torch.allclose(lin.weight.grad, ref.weight.grad, atol=1e-4)
    assert torch.allclose(lin.bias.grad, ref.bias.grad, atol=1e-5)


def test_rms_norm_module():
    kb = build_kernel_backend("b200")
    norm = kb.rms_norm(8, 1e-6)
    x = torch.randn(4, 8)
    want = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(norm(x), want, atol=1e-6)


def _sdpa(q, k, v, causal, offset, scale):
    rep = q.shape[1] // k.shape[1]
    k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    s = (q @ k.transpose(-1, -2)) * scale
    if causal:
        qp = torch.arange(q.shape[2])[:, None] + offset
        s = s.masked_fill(torch.arange(k.shape[2])[None, :] > qp, -math.inf)
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize("causal,offset", [(True, 0), (True, 6), (False, 0)])
def test_local_attention_matches_softmax_attention(causal, offset):
    torch.manual_seed(1)
    kb = build_kernel_backend("torch")
    q = torch.randn(2, 4, 10, 16, dtype=torch.float64, requires_grad=True)
    k = torch.randn(2, 2, 16, 16, dtype=torch.float64, requires_grad=True)
    v = torch.randn(2, 2, 16, 16, dtype=torch.float64, requires_grad=True)
    out = kb.local_attention(q, k, v, causal=causal, sequence_offset=offset)
    refs = [t.detach().clone().requires_grad_() for t in (q, k, v)]
    want = _sdpa(*refs, causal, offset, 0.25)
    assert out.shape == (2, 4, 10, 16)
    assert torch.allclose(out, want, atol=1e-10)
    g = torch.randn_like(out)
    out.backward(g)
    want.backward(g)
    for a, b in zip((q, k, v), refs):
        assert torch.allclose(a.grad, b.grad, atol=1e-10)
    with pytest.raises(NotImplementedError):
        kb.local_attention(q, k, v, dropout_p=0.1)
