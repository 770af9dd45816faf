"""tcgen05 attention backward (dK/dV/dQ) against fp32 autograd of the reference formula."""

import math
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.ops import functional as F  # noqa: E402


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _ref(q, k, v, q_off=0, k_off=0):
    B, S, Hq, D = q.shape
    rep = Hq // k.shape[2]
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(rep, 2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, 2).transpose(1, 2)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    qp = torch.arange(S, device=q.device) + q_off
    kp = torch.arange(k.shape[1], device=q.device) + k_off
    s = s.masked_fill(kp[None, :] > qp[:, None], float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(1, 2)


@pytest.mark.parametrize("d,hq,hkv,s,b", [(64, 4, 4, 512, 2), (128, 8, 2, 384, 1),
                                          (64, 2, 1, 200, 2), (128, 4, 4, 130, 1)])
def test_tc_backward_matches_fp32(d, hq, hkv, s, b):
    torch.manual_seed(1)
    qkv = torch.randn(s, b, hq + 2 * hkv, d, device="cuda").bfloat16()
    q = qkv[:, :, :hq].transpose(0, 1)
    k = qkv[:, :, hq:hq + hkv].transpose(0, 1)
    v = qkv[:, :, hq + hkv:].transpose(0, 1)
    o, lse = F.attention_fwd(q, k, v, causal=True)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = _ref(qr, kr, vr)
    assert _rel(o, ref) < 1e-2
    do = torch.randn_like(o)
    ref.backward(do.float())
    dqkv = torch.empty_like(qkv)
    dq = dqkv[:, :, :hq].transpose(0, 1)
    dk = dqkv[:, :, hq:hq + hkv].transpose(0, 1)
    dv = dqkv[:, :, hq + hkv:].transpose(0, 1)
    F.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, causal=True)
    torch.cuda.synchronize()
    from nano_megatron_b200.ops._ext import lib

    assert lib().attn_bwd_softmax_groups() == \
        (1 if os.environ.get("NMB_ATTN_BWD_SOFTMAX_GROUPS") == "1" else 2)
    assert _rel(dv, vr.grad) < 2e-2
    assert _rel(dk, kr.grad) < 2e-2
    assert _rel(dq, qr.grad) < 2e-2


def test_tc_backward_inverse_rope_matches_cpu_formula():
    torch.manual_seed(2)
    b, s, h, d = 1, 256, 2, 64
    q = torch.randn(b, s, h, d, device="cuda").bfloat16()
    k = torch.randn(b, s, h, d, device="cuda").bfloat16()
    v = torch.randn(b, s, h, d, device="cuda").bfloat16()
    o, lse = F.attention_fwd(q, k, v, causal=True)
    do = torch.randn_like(o)
    pos = torch.arange(s, device="cuda", dtype=torch.int32) + 3
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    outs = []
    for dev in ("cuda", "cpu"):
        args = [t.to(dev) for t in (q, k, v, o, do, lse)]
        dq, dk, dv = (torch.empty_like(args[0]), torch.empty_like(args[1]),
                      torch.empty_like(args[2]))
        F.attention_bwd(*args, dq, dk, dv, causal=True, q_pos=pos.to(dev), k_pos=pos.to(dev),
                        inv_freq=inv.to(dev))
        outs.append((dq.cpu(), dk.cpu(), dv.cpu()))
    for a, c in zip(*outs):
        assert _rel(a, c) < 2e-2


def test_one_softmax_warp_group_variant():
    """The backward with one softmax warp group per CTA (the default has two, each taking
    half of the query columns and of the dQ / dK-dV drains) passes the same checks, in a
    fresh process."""
    if os.environ.get("NMB_ATTN_BWD_SOFTMAX_GROUPS") == "1":
        pytest.skip("already running the variant")
    env = dict(os.environ, NMB_ATTN_BWD_SOFTMAX_GROUPS="1")
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-m", "gpu",
                        "-p", "no:cacheprovider", "-k", "matches_fp32 or inverse_rope"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
