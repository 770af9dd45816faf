"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.ops import gemm as G  # noqa: E402
from nano_megatron_b200.ops import lib, status_word  # noqa: E402

DEV = "cuda"


def _rel(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (4096, 1024, 1024), (300, 520, 200), (296, 520, 200),
                                   (1000, 1368, 2736), (256, 8192, 1024), (64, 64, 32)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_layouts(m, n, k, a_mn, b_mn):
    # TMA needs 16-byte row pitches: MN-major operands need M (or N) % 8 == 0.
    if (a_mn and m % 8) or (b_mn and n % 8) or k % 8:
        pytest.skip("row pitch not a multiple of 16 bytes")
    torch.manual_seed(0)
    A = torch.randn(m, k, device=DEV).bfloat16()
    B = torch.randn(n, k, device=DEV).bfloat16()
    a_store = A.t().contiguous() if a_mn else A
    b_store = B.t().contiguous() if b_mn else B
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    G.gemm(a_store, b_store, out, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert _rel(out, ref) < 1e-2
    assert int(status_word(torch.device(DEV)).item()) == 0


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_fp32_accumulate(bn):
    torch.manual_seed(1)
    M, N, K = 512, 384, 1000  # wgrad shape: [N_out, K_in] += dy^T x, tokens = 1000
    dy = torch.randn(K, M, device=DEV).bfloat16()
    x = torch.randn(K, N, device=DEV).bfloat16()
    main = torch.randn(M, N, device=DEV)
    start = main.clone()
    G.gemm(dy, x, main, a_mn=True, b_mn=True, epilogue=G.EPI_F32_ACC, beta=1.0, block_n=bn)
    torch.cuda.synchronize()
    ref = start + dy.float().t() @ x.float()
    assert _rel(main, ref) < 1e-3


def test_gemm_residual_and_alpha():
    torch.manual_seed(2)
    A = torch.randn(700, 512, device=DEV).bfloat16()
    B = torch.randn(1024, 512, device=DEV).bfloat16()
    R = torch.randn(700, 1024, device=DEV).bfloat16()
    alpha = torch.tensor([0.5], device=DEV)
    out = torch.empty(700, 1024, device=DEV, dtype=torch.bfloat16)
    G.gemm(A, B, out, residual=R, alpha_t=alpha)
    ref = 0.5 * (A.float() @ B.float().t()) + R.float()
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("ffn", [688, 1368, 2736])
def test_gemm_swiglu(ffn):
    torch.manual_seed(3)
    M, H = 777, 1024
    x = torch.randn(M, H, device=DEV).bfloat16() * 0.5
    w = (torch.randn(2 * ffn, H, device=DEV) * 0.03).bfloat16()
    h, gu = G.swiglu_fwd(x, w, ffn)
    g = x.float() @ w[:ffn].float().t()
    u = x.float() @ w[ffn:].float().t()
    assert _rel(gu[:, :ffn], g) < 1e-2
    assert _rel(gu[:, ffn:], u) < 1e-2
    assert _rel(h, torch.nn.functional.silu(g) * u) < 2e-2


@pytest.mark.parametrize("d,hq,hkv", [(64, 16, 16), (128, 8, 2)])
def test_gemm_qkv_rope(d, hq, hkv):
    torch.manual_seed(4)
    B, S, H = 2, 256, hq * d
    theta = 10000.0
    x = torch.randn(B * S, H, device=DEV).bfloat16()
    n = (hq + 2 * hkv) * d
    w = (torch.randn(n, H, device=DEV) * 0.02).bfloat16()
    pos = torch.arange(S, device=DEV, dtype=torch.int32) + 5
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, device=DEV, dtype=torch.float32) / d))
    out = G.qkv_rope_fwd(x, w, pos, inv_freq, d, (hq + hkv) * d)
    raw = (x.float() @ w.float().t()).view(B, S, hq + 2 * hkv, d)
    ang = pos.float()[:, None] * inv_freq[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[None, :, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[None, :, None, :]
    x1, x2 = raw[..., : d // 2], raw[..., d // 2:]
    rot = torch.cat([-x2, x1], -1)
    roped = raw * cos + rot * sin
    ref = torch.cat([roped[:, :, : hq + hkv], raw[:, :, hq + hkv:]], 2).reshape(B * S, n)
    assert _rel(out, ref) < 1e-2


def _attn_ref(q, k, v, causal=True, q_off=0, k_off=0):
    # q [B,S,Hq,D], k/v [B,Sk,Hkv,D] -> fp32 reference
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    rep = Hq // Hkv
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(rep, 2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, 2).transpose(1, 2)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    if causal:
        qp = torch.arange(S, device=q.device) + q_off
        kp = torch.arange(k.shape[1], device=q.device) + k_off
        s = s.masked_fill(kp[None, :] > qp[:, None], float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ vf).transpose(1, 2)


@pytest.mark.parametrize("d,hq,hkv,s,b", [(64, 4, 4, 512, 2), (128, 8, 2, 300, 1),
                                          (64, 2, 1, 1024, 1), (128, 4, 4, 128, 3)])
@pytest.mark.parametrize("fwd", ["tcgen05", "mma"])
def test_flash_attention_fwd_bwd(d, hq, hkv, s, b, fwd):
    torch.manual_seed(5)
    qkv = torch.randn(b, s, hq + 2 * hkv, d, device=DEV).bfloat16()
    q, k, v = qkv[:, :, :hq], qkv[:, :, hq:hq + hkv], qkv[:, :, hq + hkv:]
    o = torch.empty(b, s, hq, d, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(b, hq, s, device=DEV)
    scale = 1.0 / math.sqrt(d)
    if fwd == "tcgen05":
        lib().flash_attn_fwd_tc(q, k, v, o, lse, scale, True, 0, 0,
                                status_word(torch.device(DEV)))
    else:
        lib().flash_attn_fwd(q, k, v, o, lse, scale, True, 0, 0)
    qr = q.detach().float().requires_grad_()
    kr = k.detach().float().requires_grad_()
    vr = v.detach().float().requires_grad_()
    ref = _attn_ref(qr, kr, vr)
    assert _rel(o, ref) < 1e-2
    do = torch.randn_like(o)
    ref.backward(do.float())
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = dqkv[:, :, :hq], dqkv[:, :, hq:hq + hkv], dqkv[:, :, hq + hkv:]
    delta = torch.empty(b * hq * s, device=DEV)
    dq_acc = torch.empty(b * s * hq * d, device=DEV)
    lib().flash_attn_bwd(q, k, v, o, do, lse, dq, dk, dv, delta, dq_acc, scale, True, 0, 0,
                         None, None, None)
    torch.cuda.synchronize()
    assert _rel(dv, vr.grad) < 2e-2
    assert _rel(dk, kr.grad) < 2e-2
    assert _rel(dq, qr.grad) < 2e-2


def test_flash_attention_offsets_noncausal():
    torch.manual_seed(6)
    b, s, sk, hq, hkv, d = 1, 256, 512, 4, 2, 64
    q = torch.randn(b, s, hq, d, device=DEV).bfloat16()
    k = torch.randn(b, sk, hkv, d, device=DEV).bfloat16()
    v = torch.randn(b, sk, hkv, d, device=DEV).bfloat16()
    o = torch.empty_like(q)
    lse = torch.empty(b, hq, s, device=DEV)
    st = status_word(torch.device(DEV))
    for fn in (lambda *a: lib().flash_attn_fwd(*a), lambda *a: lib().flash_attn_fwd_tc(*a, st)):
        fn(q, k, v, o, lse, 1 / 8.0, True, 256, 0)
        assert _rel(o, _attn_ref(q, k, v, True, 256, 0)) < 1e-2
        fn(q, k, v, o, lse, 1 / 8.0, False, 0, 0)
        assert _rel(o, _attn_ref(q, k, v, False)) < 1e-2
        fn(q, k, v, o, lse, 1 / 8.0, True, 0, 300)  # keys beyond every query: empty rows
        assert o.float().abs().max().item() == 0.0
    assert int(st.item()) == 0


@pytest.mark.parametrize("h", [256, 1024, 2048, 4096])
def test_rmsnorm(h):
    torch.manual_seed(7)
    x = torch.randn(1000, h, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(h, device=DEV)).bfloat16()
    y = torch.empty_like(x)
    rstd = torch.empty(1000, device=DEV)
    lib().rmsnorm_fwd(x, w, y, rstd, 1e-5)
    xr = x.float().requires_grad_()
    wr = w.float().requires_grad_()
    ref = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    assert _rel(y, ref) < 1e-2
    dy = torch.randn_like(x)
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(h, device=DEV)
    lib().rmsnorm_bwd(x, w, dy, rstd, dx, dw, None)
    assert _rel(dx, xr.grad) < 1e-2
    assert _rel(dw, wr.grad) < 1e-2


def test_swiglu_bwd_and_embedding_and_ce():
    torch.manual_seed(8)
    T, F = 513, 688
    gu = torch.randn(T, 2 * F, device=DEV).bfloat16()
    dh = torch.randn(T, F, device=DEV).bfloat16()
    g = gu[:, :F].float().requires_grad_()
    u = gu[:, F:].float().requires_grad_()
    (torch.nn.functional.silu(g) * u).backward(dh.float())
    dgu = torch.empty_like(gu)
    lib().swiglu_bwd(gu, dh, dgu)
    assert _rel(dgu[:, :F], g.grad) < 1e-2 and _rel(dgu[:, F:], u.grad) < 1e-2

    V, H = 1000, 256
    w = torch.randn(V, H, device=DEV).bfloat16()
    ids = torch.randint(0, 2 * V, (T,), device=DEV)
    out = torch.empty(T, H, device=DEV, dtype=torch.bfloat16)
    lib().embedding_fwd(ids, w, V, out)  # shard [V, 2V)
    mask = (ids >= V) & (ids < 2 * V)
    ref = torch.zeros(T, H, device=DEV)
    ref[mask] = w[(ids - V)[mask]].float()
    assert torch.equal(out.float(), ref)
    grad = torch.zeros(V, H, device=DEV)
    dy = torch.randn(T, H, device=DEV).bfloat16()
    lib().embedding_bwd(ids, dy, grad, V)
    refg = torch.zeros(V, H, device=DEV).index_add_(0, (ids - V)[mask], dy.float()[mask])
    assert _rel(grad, refg) < 1e-5

    Vc = 8192
    logits = torch.randn(T, Vc, device=DEV).bfloat16() * 3
    labels = torch.randint(0, Vc, (T,), device=DEV)
    labels[::7] = -100
    lg = logits.float().requires_grad_()
    ref_loss = torch.nn.functional.cross_entropy(lg, labels, ignore_index=-100, reduction="sum")
    ref_loss.backward()
    loss_row = torch.empty(T, device=DEV)
    work = logits.clone()
    lib().ce_fused(work, labels, loss_row, True)
    assert abs(loss_row.sum().item() - ref_loss.item()) / abs(ref_loss.item()) < 1e-3
    assert _rel(work, lg.grad) < 1e-2
    # two shards through stats/finish
    halves = [logits[:, : Vc // 2].clone(), logits[:, Vc // 2:].clone()]
    stats = torch.empty(2, T, 3, device=DEV)
    for r in range(2):
        lib().ce_stats(halves[r], labels, r * Vc // 2, stats[r])
    losses = []
    for r in range(2):
        lr = torch.empty(T, device=DEV)
        lib().ce_finish(halves[r], labels, r * Vc // 2, stats, 2, lr, True)
        losses.append(lr)
    assert abs(losses[0].sum().item() - ref_loss.item()) / abs(ref_loss.item()) < 1e-3
    assert _rel(torch.cat(halves, 1), lg.grad) < 1e-2


def test_adamw_matches_torch():
    torch.manual_seed(9)
    n = 10007
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    pb = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    for step in range(1, 4):
        ref.grad = g.clone()
        opt.step()
        lib().adamw_step(p, g, m, v, pb, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, None, None)
    assert _rel(p, ref.detach()) < 1e-6
    assert _rel(pb, ref.detach()) < 1e-2
    parts = lib().sumsq_partials(g)
    assert abs(parts.sum().item() - g.pow(2).sum().item()) / g.pow(2).sum().item() < 1e-5


def test_philox_dropout_statistics_and_replay():
    """Keep rate ~ 1-p, kept values scaled by 1/(1-p), the mask replays bit-exactly from the
    seed (so backward needs no stored mask), and different seeds give different masks."""
    from nano_megatron_b200.nn.dropout import DropoutMask

    x = torch.ones(1 << 20, device=DEV, dtype=torch.bfloat16)
    p = 0.1
    d = DropoutMask(p, seed=1234)
    y = d(x)
    kept = (y != 0).float().mean().item()
    assert abs(kept - (1 - p)) < 3e-3
    assert torch.allclose(y[y != 0].float(), torch.full_like(y[y != 0].float(), 1 / (1 - p)),
                          rtol=1e-2)
    g = d.backward(x)
    assert torch.equal(g, y)                      # same mask from (seed, index)
    y2 = DropoutMask(p, seed=1235)(x)
    assert not torch.equal(y2 != 0, y != 0)


@pytest.mark.parametrize("vocab", [8192, 1000])
def test_lm_head_ce_statistics_epilogue_matches_fp32(vocab):
    """LM head GEMM whose epilogue writes per-tile (max, sum exp), then the one-pass
    cross-entropy: loss rows and the in-place softmax - onehot gradient against fp32 torch
    (a vocabulary that is not a multiple of the 256-column tile covers the tail tile;
    ignored rows carry label -100)."""
    from nano_megatron_b200.ops import functional as F

    torch.manual_seed(11)
    m, h = 512, 256
    x = torch.randn(m, h, device=DEV).bfloat16()
    w = (torch.randn(vocab, h, device=DEV) * 0.1).bfloat16()
    labels = torch.randint(0, vocab, (m,), device=DEV)
    labels[::7] = -100
    logits, rows = F.linear_ce(x, w, labels, write_grad=True)
    torch.cuda.synchronize()
    assert int(status_word(x.device).item()) == 0
    ref_logits = x.float() @ w.float().t()
    valid = labels >= 0
    lse = torch.logsumexp(ref_logits, -1)
    tgt = ref_logits.gather(1, labels.clamp_min(0)[:, None])[:, 0]
    ref_rows = torch.where(valid, lse - tgt, torch.zeros_like(lse))
    assert _rel(rows, ref_rows) < 1e-2
    grad = torch.softmax(ref_logits, -1)
    grad[torch.arange(m, device=DEV)[valid], labels[valid]] -= 1.0
    grad[~valid] = 0.0
    assert _rel(logits, grad) < 2e-2
