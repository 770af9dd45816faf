"""Fused TP collectives (AG->GEMM, GEMM->RS) against fp32 PyTorch references.

The TP ranks are emulated inside one process on one GPU: every "peer" buffer
is a local allocation and the ranks' kernels are issued phase by phase (all
publishes/GEMMs first, then the consumers), so every flag a kernel waits on is
already set when it runs -- no kernel ever waits on one launched after it. The
real multi-process path (IPC-mapped peers on several GPUs) is covered by
``test_comm_gemm_multigpu.py``.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.distributed.symmetric import SymmetricWorkspace  # noqa: E402
from nano_megatron_b200.ops import comm_gemm as CG  # noqa: E402
from nano_megatron_b200.ops import functional as F  # noqa: E402
from nano_megatron_b200.ops._ext import status_word  # noqa: E402

DEV = torch.device("cuda")
MB = 1 << 20


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _ok():
    torch.cuda.synchronize()
    assert int(status_word(DEV).item()) == 0


@pytest.mark.parametrize("tp", [2, 4])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("K", [512, 1368])
def test_gemm_reduce_scatter(tp, b_mn, K):
    """K = 1368: the down projection's reduction width at TP2 (a partial last K block)."""
    torch.manual_seed(tp)
    ws = SymmetricWorkspace.emulated(tp, rs_bytes=16 * MB, ag_bytes=8 * MB, device=DEV)
    R, N = 256, 384
    M = R * tp
    for it in range(3):  # exercises both parities and epoch advance
        a = [torch.randn(M, K, device=DEV).bfloat16() for _ in range(tp)]
        w = [torch.randn(N, K, device=DEV).bfloat16() for _ in range(tp)]
        res = [torch.randn(R, N, device=DEV).bfloat16() for _ in range(tp)]
        bstore = [x.t().contiguous() if b_mn else x for x in w]
        for r in range(tp):
            CG.rs_issue(ws[r], a[r], bstore[r], b_mn=b_mn)
        outs = [torch.empty(R, N, device=DEV, dtype=torch.bfloat16) for _ in range(tp)]
        for r in range(tp):
            CG.rs_finish(ws[r], outs[r], res[r])
        _ok()
        full = sum(a[r].float() @ w[r].float().t() for r in range(tp))
        for r in range(tp):
            ref = full[r * R:(r + 1) * R] + res[r].float()
            assert _rel(outs[r], ref) < 1e-2, (it, r)


@pytest.mark.parametrize("tp", [2, 4])
def test_allgather_gemm_bf16_and_gathered_copy(tp):
    torch.manual_seed(10 + tp)
    ws = SymmetricWorkspace.emulated(tp, rs_bytes=2 * MB, ag_bytes=8 * MB, device=DEV)
    R, K, N = 256, 576, 640
    for it in range(3):
        x = [torch.randn(R, K, device=DEV).bfloat16() for _ in range(tp)]
        w = torch.randn(N, K, device=DEV).bfloat16()
        for r in range(tp):
            CG.ag_issue(ws[r], x[r])
        outs, xf = [], []
        for r in range(tp):
            o = torch.empty(R * tp, N, device=DEV, dtype=torch.bfloat16)
            g = torch.empty(R * tp, K, device=DEV, dtype=torch.bfloat16)
            CG.ag_finish(ws[r], x[r], w, o, xfull=g)
            outs.append(o)
            xf.append(g)
        _ok()
        xcat = torch.cat(x)
        ref = xcat.float() @ w.float().t()
        for r in range(tp):
            assert torch.equal(xf[r], xcat), (it, r)
            assert _rel(outs[r], ref) < 1e-2, (it, r)


@pytest.mark.parametrize("n_local", [512, 1368])
def test_allgather_gemm_dgrad_layout(n_local):
    """dgrad of a row-parallel layer: A = dy (gathered), B = W stored [N_local, K] (MN-major);
    1368 = the 311M model's local FFN width at TP2 (a partial last output tile)."""
    tp, R, K = 2, 384, 1024
    ws = SymmetricWorkspace.emulated(tp, rs_bytes=2 * MB, ag_bytes=8 * MB, device=DEV)
    dy = [torch.randn(R, K, device=DEV).bfloat16() for _ in range(tp)]
    w = torch.randn(K, n_local, device=DEV).bfloat16()       # weight [out=K, in_local]
    for r in range(tp):
        CG.ag_issue(ws[r], dy[r])
    outs = []
    for r in range(tp):
        o = torch.empty(R * tp, n_local, device=DEV, dtype=torch.bfloat16)
        CG.ag_finish(ws[r], dy[r], w, o, b_mn=True)
        outs.append(o)
    _ok()
    ref = torch.cat(dy).float() @ w.float()
    for o in outs:
        assert _rel(o, ref) < 1e-2


@pytest.mark.parametrize("ffn", [768, 344, 1368])
def test_allgather_gemm_rope_and_swiglu_match_local_kernels(ffn):
    """``ffn`` = the local SwiGLU width; 344 and 1368 (F = 688 / 2736 at TP2) are not
    multiples of the 128-column output tile."""
    tp, R, H, D = 2, 256, 512, 64
    hq, hkv = 8, 4
    ws = SymmetricWorkspace.emulated(tp, rs_bytes=2 * MB, ag_bytes=8 * MB, device=DEV)
    torch.manual_seed(3)
    x = [torch.randn(R, H, device=DEV).bfloat16() for _ in range(tp)]
    xcat = torch.cat(x)
    wqkv = (torch.randn((hq + 2 * hkv) * D, H, device=DEV) * 0.05).bfloat16()
    B = 4
    pos = torch.arange(R * tp // B, device=DEV, dtype=torch.int32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    ref = F.qkv_rope_linear(xcat, wqkv, pos, inv, D, (hq + hkv) * D, pos_div=B)
    for r in range(tp):
        CG.ag_issue(ws[r], x[r])
    for r in range(tp):
        o = torch.empty(R * tp, wqkv.shape[0], device=DEV, dtype=torch.bfloat16)
        CG.ag_finish(ws[r], x[r], wqkv, o, epi="rope", positions=pos, inv_freq=inv,
                     head_dim=D, rope_cols=(hq + hkv) * D, pos_div=B)
        _ok()
        assert _rel(o, ref) < 1e-3
    wgu = (torch.randn(2 * ffn, H, device=DEV) * 0.05).bfloat16()
    h_ref, gu_ref = F.swiglu_linear(xcat, wgu, ffn)
    for r in range(tp):
        CG.ag_issue(ws[r], x[r])
    for r in range(tp):
        h = torch.empty(R * tp, ffn, device=DEV, dtype=torch.bfloat16)
        gu = torch.empty(R * tp, 2 * ffn, device=DEV, dtype=torch.bfloat16)
        CG.ag_finish(ws[r], x[r], wgu, h, epi="swiglu", aux=gu, swiglu_up_row=ffn)
        _ok()
        assert _rel(h, h_ref) < 1e-3 and _rel(gu, gu_ref) < 1e-3


def test_missing_peer_times_out_with_status():
    """A peer that never publishes: the bounded wait gives up (~2 s), records 0x301 and
    the kernel returns; the context stays usable."""
    tp, R, K, N = 2, 128, 256, 256
    ws = SymmetricWorkspace.emulated(tp, rs_bytes=2 * MB, ag_bytes=2 * MB, device=DEV)
    x = torch.randn(R, K, device=DEV).bfloat16()
    w = torch.randn(N, K, device=DEV).bfloat16()
    CG.ag_issue(ws[0], x)                  # rank 1 never publishes this epoch
    o = torch.empty(R * tp, N, device=DEV, dtype=torch.bfloat16)
    CG.ag_finish(ws[0], x, w, o)
    torch.cuda.synchronize()
    st = status_word(DEV)
    assert int(st.item()) == 0x301
    st.zero_()
    y = torch.randn(64, 64, device=DEV) @ torch.randn(64, 64, device=DEV)  # context still fine
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()


def _aux_ws(tp, R, H):
    return SymmetricWorkspace.emulated(tp, rs_bytes=2 * MB, ag_bytes=R * H * 2, device=DEV,
                                       emb_bytes=R * H * 2, ce_bytes=tp * tp * R * 12)


@pytest.mark.parametrize("tp", [2, 4])
def test_embedding_lookup_scatter_matches_full_lookup(tp):
    """Each rank stores only the rows of its vocabulary shard into the sequence owners'
    slots; every rank's output equals a plain lookup of its own tokens."""
    torch.manual_seed(20 + tp)
    V, H, R = 512, 256, 128
    Vl = V // tp
    ws = _aux_ws(tp, R, H)
    w = torch.randn(V, H, device=DEV).bfloat16()
    for it in range(3):                    # parities and epoch advance
        ids = torch.randint(0, V, (R * tp,), device=DEV)
        for r in range(tp):
            CG.embedding_issue(ws[r], ids, w[r * Vl:(r + 1) * Vl].contiguous(), r * Vl)
        outs = [torch.empty(R, H, device=DEV, dtype=torch.bfloat16) for _ in range(tp)]
        for r in range(tp):
            CG.embedding_finish(ws[r], outs[r])
        _ok()
        for r in range(tp):
            assert torch.equal(outs[r], w[ids[r * R:(r + 1) * R]]), (it, r)


@pytest.mark.parametrize("tp", [2, 4])
def test_embedding_backward_gather_matches_scatter_add(tp):
    torch.manual_seed(30 + tp)
    V, H, R = 512, 256, 128
    Vl = V // tp
    ws = _aux_ws(tp, R, H)
    ids = torch.randint(0, V, (R * tp,), device=DEV)
    dy = [torch.randn(R, H, device=DEV).bfloat16() for _ in range(tp)]
    grads = [torch.zeros(Vl, H, device=DEV) for _ in range(tp)]
    for r in range(tp):
        CG.ag_issue(ws[r], dy[r])
    for r in range(tp):
        CG.embedding_bwd_finish(ws[r], ids, dy[r], grads[r], r * Vl)
    _ok()
    ref = torch.zeros(V, H, device=DEV).index_add_(0, ids, torch.cat(dy).float())
    for r in range(tp):
        torch.testing.assert_close(grads[r], ref[r * Vl:(r + 1) * Vl], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tp", [2, 4])
def test_vocab_parallel_ce_by_peer_stores_matches_fp32(tp):
    """Row statistics exchanged by peer stores + flag: loss rows and the in-place
    softmax - onehot gradient equal fp32 cross-entropy over the full vocabulary."""
    torch.manual_seed(40 + tp)
    T, V = 256, 1024
    Vl = V // tp
    ws = _aux_ws(tp, T // tp, 64)
    full = (torch.randn(T, V, device=DEV) * 3).bfloat16()
    labels = torch.randint(0, V, (T,), device=DEV)
    labels[::7] = -100
    for it in range(2):
        shards = [full[:, r * Vl:(r + 1) * Vl].contiguous() for r in range(tp)]
        for r in range(tp):
            CG.ce_issue(ws[r], shards[r], labels, r * Vl)
        rows = [CG.ce_finish(ws[r], shards[r], labels, r * Vl, write_grad=True)
                for r in range(tp)]
        _ok()
        ref = torch.nn.functional.cross_entropy(full.float(), labels, ignore_index=-100,
                                                reduction="none")
        valid = labels >= 0
        onehot = torch.zeros(T, V, device=DEV)
        onehot[valid, labels[valid]] = 1.0
        gref = (full.float().softmax(-1) - onehot) * valid[:, None]
        for r in range(tp):
            torch.testing.assert_close(rows[r], ref, rtol=2e-3, atol=2e-3)
            assert _rel(shards[r], gref[:, r * Vl:(r + 1) * Vl]) < 1e-2, (it, r)
