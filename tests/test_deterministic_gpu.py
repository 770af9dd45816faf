"""Deterministic kernel mode: every reduction that otherwise uses fp32 atomics runs in a
fixed order, so repeated runs are bitwise equal. Each kernel is also checked against a
plain PyTorch fp32 reference of the same op, and against the default (atomic) mode."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.ops import functional as F  # noqa: E402
from nano_megatron_b200.ops import gemm as G  # noqa: E402
from nano_megatron_b200.ops import lib, status_word  # noqa: E402
from nano_megatron_b200.ops.deterministic import deterministic, is_deterministic  # noqa: E402

DEV = "cuda"


def _rel(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def test_switch_reaches_the_kernel_library():
    assert not is_deterministic() and not lib().get_deterministic()
    with deterministic():
        assert is_deterministic() and lib().get_deterministic()
    assert not lib().get_deterministic()


@pytest.mark.parametrize("n", [4096, 1001])
def test_slots_sum_adds_slots_in_order(n):
    torch.manual_seed(0)
    slots = torch.randn(5, n, device=DEV) * torch.logspace(-3, 3, 5, device=DEV)[:, None]
    out = torch.randn(n, device=DEV)
    want = out.clone()
    for s in range(5):
        want = want + slots[s]
    lib().slots_sum(slots, out, True)
    assert torch.equal(out, want)
    fresh = torch.zeros(n, device=DEV)
    for s in range(5):
        fresh = fresh + slots[s]
    lib().slots_sum(slots, out, False)
    assert torch.equal(out, fresh)


def test_wgrad_runs_unsplit_and_is_bitwise_reproducible():
    torch.manual_seed(1)
    M, N, K = 256, 256, 8192  # split-K would cut these 4 tiles 8 ways
    dy = torch.randn(K, M, device=DEV).bfloat16()
    x = torch.randn(K, N, device=DEV).bfloat16()
    start = torch.randn(M, N, device=DEV)
    ref = start + dy.float().t() @ x.float()
    outs = []
    with deterministic():
        for _ in range(3):
            main = start.clone()
            G.linear_wgrad(dy, x, main)
            outs.append(main)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert _rel(outs[0], ref) < 1e-3


@pytest.mark.parametrize("h", [1024, 2048])
def test_rmsnorm_weight_gradient_fixed_order(h):
    torch.manual_seed(2)
    rows = 3000
    x = torch.randn(rows, h, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(h, device=DEV)).bfloat16()
    dy = torch.randn_like(x)
    _, rstd = F.rmsnorm(x, w, 1e-5)
    xr = x.float().requires_grad_()
    wr = w.float().requires_grad_()
    ref = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    ref.backward(dy.float())
    dw_atomic = torch.full((h,), 0.5, device=DEV)
    dx_atomic = F.rmsnorm_bwd(x, w, dy, rstd, dw_atomic)
    runs = []
    with deterministic():
        for _ in range(3):
            dw = torch.full((h,), 0.5, device=DEV)
            dx = F.rmsnorm_bwd(x, w, dy, rstd, dw)
            runs.append((dx, dw))
    torch.cuda.synchronize()
    for dx, dw in runs[1:]:
        assert torch.equal(dw, runs[0][1])
        assert torch.equal(dx, runs[0][0])
    assert torch.equal(runs[0][0], dx_atomic)  # dx never used atomics
    assert _rel(runs[0][1] - 0.5, wr.grad) < 1e-2
    assert _rel(runs[0][1], dw_atomic) < 1e-5


def test_embedding_backward_sorted_runs():
    torch.manual_seed(3)
    T, H, V, vstart = 5000, 256, 64, 32  # few ids: long runs of repeated tokens
    ids = torch.randint(0, 128, (T,), device=DEV)
    dy = torch.randn(T, H, device=DEV).bfloat16()
    base = torch.randn(V, H, device=DEV)
    local = ids - vstart
    mask = (local >= 0) & (local < V)
    ref = base.clone().index_add_(0, local[mask], dy[mask].float())
    atomic = base.clone()
    F.embedding_bwd(ids, dy, atomic, vstart)
    runs = []
    with deterministic():
        for _ in range(3):
            g = base.clone()
            F.embedding_bwd(ids, dy, g, vstart)
            runs.append(g)
    torch.cuda.synchronize()
    assert all(torch.equal(runs[0], g) for g in runs[1:])
    assert _rel(runs[0], ref) < 1e-6
    assert _rel(runs[0], atomic) < 1e-6


def _attn_ref(q, k, v, causal=True):
    rep = q.shape[2] // k.shape[2]
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(rep, 2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, 2).transpose(1, 2)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        n = q.shape[1]
        s = s.masked_fill(torch.ones(n, n, device=q.device, dtype=torch.bool).triu(1), -math.inf)
    return (torch.softmax(s, -1) @ vf).transpose(1, 2)


@pytest.mark.parametrize("d,hq,hkv,s,causal", [(64, 4, 2, 512, True), (128, 4, 4, 640, True),
                                               (64, 2, 2, 384, False)])
def test_attention_backward_dq_slots(d, hq, hkv, s, causal):
    torch.manual_seed(4)
    b = 2
    q = torch.randn(b, s, hq, d, device=DEV).bfloat16()
    k = torch.randn(b, s, hkv, d, device=DEV).bfloat16()
    v = torch.randn(b, s, hkv, d, device=DEV).bfloat16()
    o, lse = F.attention_fwd(q, k, v, causal=causal)
    do = torch.randn_like(o)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    _attn_ref(qr, kr, vr, causal).backward(do.float())

    def grads():
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        F.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, causal=causal)
        return dq, dk, dv

    atomic = grads()
    with deterministic():
        runs = [grads() for _ in range(3)]
    torch.cuda.synchronize()
    for r in runs[1:]:
        for a, bb in zip(runs[0], r):
            assert torch.equal(a, bb)
    for got, want in zip(runs[0], (qr.grad, kr.grad, vr.grad)):
        assert _rel(got, want) < 2e-2
    for got, want in zip(runs[0], atomic):
        assert _rel(got, want) < 5e-3
    assert int(status_word(torch.device(DEV)).item()) == 0


def _train(deterministic_mode: bool, steps: int = 2):
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components

    cfg = config_from_dict({
        "model": {"layers": 2, "hidden_size": 256, "ffn_hidden_size": 688, "heads": 4,
                  "kv_heads": 2, "seq_length": 512, "vocab_size": 1024},
        "distributed": {"device": "cuda", "backend": "nccl"},
        "kernels": {"backend": "b200", "cuda_graphs": True,
                    "deterministic": deterministic_mode},
        "training": {"micro_batch_size": 4, "gradient_accumulation_steps": 2, "seed": 21},
        "optimizer": {"lr": 1e-3, "clip_grad_norm": 1.0}})
    rt = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, rt)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    g = torch.Generator().manual_seed(9)
    losses = []
    for _ in range(steps):
        ids = torch.randint(0, 1024, (8, 513), generator=g)
        out = tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        losses.append((out["loss_sum"] / out["token_count"]).detach().clone())
    torch.cuda.synchronize()
    params = {n: p.detach().clone() for n, p in comps.model.named_parameters()}
    grads = {n: p.main_grad.detach().clone() for n, p in comps.model.named_parameters()}
    return losses, params, grads


def test_training_steps_are_bitwise_reproducible_in_deterministic_mode():
    """Two fresh runs of two optimizer steps (CUDA graphs on, gradient accumulation 2,
    4 key blocks per attention row, repeated tokens in the embedding backward): loss,
    parameters and gradients bitwise equal; and within fp32/bf16 rounding of the default
    mode."""
    try:
        a = _train(True)
        b = _train(True)
    finally:
        from nano_megatron_b200.ops.deterministic import set_deterministic

        set_deterministic(False)
    for la, lb in zip(a[0], b[0]):
        assert torch.equal(la, lb)
    for n in a[1]:
        assert torch.equal(a[1][n], b[1][n]), n
        assert torch.equal(a[2][n], b[2][n]), n
    default = _train(False)
    for la, ld in zip(a[0], default[0]):
        assert abs(float(la) - float(ld)) < 1e-2 * abs(float(ld))
