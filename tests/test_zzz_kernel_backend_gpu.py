"""The kernel-backend seam on a B200: linear (tcgen05 GEMMs), RMSNorm and local attention
(tcgen05 flash attention) in bf16 against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.nn.kernels import build_kernel_backend  # noqa: E402

DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_linear_runs_the_gemm_kernels():
    torch.manual_seed(0)
    kb = build_kernel_backend("b200")
    lin = kb.linear(1024, 512, bias=True).to(DEV, torch.bfloat16)
    w, b = lin.weight.detach().float(), lin.bias.detach().float()
    x = torch.randn(2, 128, 1024, device=DEV).bfloat16().requires_grad_()
    y = lin(x)
    xr = x.detach().float().requires_grad_()
    wr, br = w.clone().requires_grad_(), b.clone().requires_grad_()
    yr = xr @ wr.t() + br
    assert _rel(y, yr) < 1e-2
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g.float())
    torch.cuda.synchronize()
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(lin.weight.grad, wr.grad) < 1e-2
    assert _rel(lin.bias.grad, br.grad) < 1e-2


def test_rms_norm_module_on_cuda():
    kb = build_kernel_backend("b200")
    norm = kb.rms_norm(1024, 1e-5, device=DEV, dtype=torch.bfloat16)
    x = torch.randn(64, 1024, device=DEV).bfloat16()
    want = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5)
    assert _rel(norm(x), want) < 1e-2


def _ref(q, k, v, causal, offset):
    rep = q.shape[1] // k.shape[1]
    k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        qp = torch.arange(q.shape[2], device=q.device)[:, None] + offset
        s = s.masked_fill(torch.arange(k.shape[2], device=q.device)[None, :] > qp, -math.inf)
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize("sq,causal,offset", [(256, True, 0), (256, False, 0), (128, True, 128)])
def test_local_attention_runs_the_flash_kernels(sq, causal, offset):
    torch.manual_seed(1)
    kb = build_kernel_backend("b200")
    q = torch.randn(2, 4, sq, 64, device=DEV).bfloat16().requires_grad_()
    k = torch.randn(2, 2, 256, 64, device=DEV).bfloat16().requires_grad_()
    v = torch.randn(2, 2, 256, 64, device=DEV).bfloat16().requires_grad_()
    out = kb.local_attention(q, k, v, causal=causal, sequence_offset=offset)
    refs = [t.detach().float().requires_grad_() for t in (q, k, v)]
    want = _ref(*refs, causal, offset)
    assert _rel(out, want) < 1e-2
    g = torch.randn_like(out)
    out.backward(g)
    want.backward(g.float())
    torch.cuda.synchronize()
    for a, b in zip((q, k, v), refs):
        assert _rel(a.grad, b.grad) < 2e-2
