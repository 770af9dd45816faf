"""Kernel microbenchmarks: CUDA-event timing of each sm_100a kernel vs its library baseline.

    python -m nano_megatron_b200.ops.bench_kernels [--case all|gemm|gemm_tiles|gemm_layer|attn|mem] [--iters N]

Prints one JSON object of achieved TFLOP/s (GEMM, attention) or GB/s and the fraction of
the measured copy bandwidth (memory-bound kernels: RMSNorm, SwiGLU backward, attention
backward prep / dQ conversion, embedding, AdamW). ``--case gemm_tiles`` sweeps the GEMM
tile width (``block_n`` 128 and 256) on the 311M model's shapes, the data behind the tile
choice in ``choose_bn`` (csrc/gemm_tcgen05.cu); ``--case attn_trace[:d128]`` prints the attention backward's in-kernel phase
times; ``--case gemm_layer`` times the layer's
GEMMs with their fused epilogues (RoPE, SwiGLU, residual) against the plain product. Also the small, self-contained workload used for ncu captures
(``--case gemm_profile`` / ``gemm_epi_profile:<swiglu|rope|residual>`` / ``attn_profile[:d128]``
run a few launches of one kernel).
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from . import functional as F
from . import gemm as G
from ._ext import lib


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def gemm_cases(iters: int) -> dict:
    res = {}
    for m, n, k in [(4096, 3072, 1024), (4096, 1024, 1024), (4096, 1024, 2736),
                    (4096, 8192, 1024), (8192, 8192, 8192)]:
        a = torch.randn(m, k, device="cuda").bfloat16()
        b = torch.randn(n, k, device="cuda").bfloat16()
        c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        fl = 2 * m * n * k
        res[f"fwd_{m}x{n}x{k}"] = fl / _time(lambda: G.gemm(a, b, c), iters) / 1e9
        res[f"cublas_{m}x{n}x{k}"] = fl / _time(lambda: torch.matmul(a, b.t(), out=c), iters) / 1e9
        bt = b.t().contiguous()
        res[f"dgrad_{m}x{n}x{k}"] = fl / _time(lambda: G.gemm(a, bt, c, b_mn=True), iters) / 1e9
        at = a.t().contiguous()
        cf = torch.zeros(m, n, device="cuda")
        res[f"wgrad_{m}x{n}x{k}"] = fl / _time(
            lambda: G.gemm(at, bt, cf, a_mn=True, b_mn=True, epilogue=G.EPI_F32_ACC, beta=1.0),
            iters) / 1e9
    # weight gradients of the 311M layers: dW[N_out, K_in] = dY^T X over 4096 tokens
    for m, n, k in [(1024, 1024, 4096), (3072, 1024, 4096), (5472, 1024, 4096),
                    (1024, 2736, 4096)]:
        dy = torch.randn(k, m, device="cuda").bfloat16()
        x = torch.randn(k, n, device="cuda").bfloat16()
        cf = torch.zeros(m, n, device="cuda")
        cb = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        fl = 2 * m * n * k
        res[f"wgrad_model_{m}x{n}x{k}"] = fl / _time(
            lambda: G.gemm(dy, x, cf, a_mn=True, b_mn=True, epilogue=G.EPI_F32_ACC, beta=1.0),
            iters) / 1e9
        res[f"cublas_wgrad_{m}x{n}x{k}"] = fl / _time(
            lambda: torch.matmul(dy.t(), x, out=cb), iters) / 1e9
    return res


def gemm_tile_cases(iters: int) -> dict:
    """TFLOP/s of forward, data-gradient and weight-gradient GEMMs at both tile widths."""
    res = {}
    for m, n, k in [(4096, 3072, 1024), (4096, 1024, 1024), (4096, 1024, 2736),
                    (4096, 5472, 1024), (4096, 8192, 1024)]:
        a = torch.randn(m, k, device="cuda").bfloat16()
        b = torch.randn(n, k, device="cuda").bfloat16()
        bt = b.t().contiguous()
        c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        fl = 2 * m * n * k
        for bn in (128, 256):
            res[f"fwd_bn{bn}_{m}x{n}x{k}"] = fl / _time(
                lambda: G.gemm(a, b, c, block_n=bn), iters) / 1e9
            res[f"dgrad_bn{bn}_{m}x{n}x{k}"] = fl / _time(
                lambda: G.gemm(a, bt, c, b_mn=True, block_n=bn), iters) / 1e9
        res[f"cublas_{m}x{n}x{k}"] = fl / _time(lambda: torch.matmul(a, b.t(), out=c), iters) / 1e9
    for m, n, k in [(1024, 1024, 4096), (3072, 1024, 4096), (5472, 1024, 4096),
                    (1024, 2736, 4096)]:
        dy = torch.randn(k, m, device="cuda").bfloat16()
        x = torch.randn(k, n, device="cuda").bfloat16()
        cf = torch.zeros(m, n, device="cuda")
        fl = 2 * m * n * k
        for bn in (128, 256):
            res[f"wgrad_bn{bn}_{m}x{n}x{k}"] = fl / _time(
                lambda: G.gemm(dy, x, cf, a_mn=True, b_mn=True, epilogue=G.EPI_F32_ACC,
                               beta=1.0, block_n=bn), iters) / 1e9
    return res


def gemm_layer_cases(iters: int, m: int = 8192) -> dict:
    """TFLOP/s of the 311M layer's GEMMs with the epilogues the model runs (RoPE on the
    QKV projection, SwiGLU on gate/up, residual add on the output and down projections),
    next to the plain product and cuBLAS at the same shape (``m`` tokens per call)."""
    res = {}
    hid, ffn, seq, hd = 1024, 2736, 512, 64
    x = torch.randn(m, hid, device="cuda").bfloat16()
    pos = torch.arange(seq, device="cuda", dtype=torch.int32)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device="cuda").float() / hd))
    w_qkv = torch.randn(3 * hid, hid, device="cuda").bfloat16()
    qkv = torch.empty(m, 3 * hid, device="cuda", dtype=torch.bfloat16)
    fl = 2 * m * 3 * hid * hid
    # rows are sequence-major (row = s * batch + b), as the model lays out a micro-batch
    res["qkv_rope"] = fl / _time(lambda: G.qkv_rope_fwd(x, w_qkv, pos, inv_freq, hd, 2 * hid,
                                                         pos_div=m // seq, out=qkv), iters) / 1e9
    res["qkv_plain"] = fl / _time(lambda: G.gemm(x, w_qkv, qkv), iters) / 1e9
    res["qkv_cublas"] = fl / _time(lambda: torch.matmul(x, w_qkv.t(), out=qkv), iters) / 1e9
    w_gu = torch.randn(2 * ffn, hid, device="cuda").bfloat16()
    h = torch.empty(m, ffn, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(m, 2 * ffn, device="cuda", dtype=torch.bfloat16)
    fl = 2 * m * 2 * ffn * hid
    res["gate_up_swiglu"] = fl / _time(lambda: G.swiglu_fwd(x, w_gu, ffn, out=h, gate_up=gu),
                                       iters) / 1e9
    res["gate_up_plain"] = fl / _time(lambda: G.gemm(x, w_gu, gu), iters) / 1e9
    res["gate_up_cublas"] = fl / _time(lambda: torch.matmul(x, w_gu.t(), out=gu), iters) / 1e9
    for name, k in (("out_proj", hid), ("down_proj", ffn)):
        a = torch.randn(m, k, device="cuda").bfloat16()
        w = torch.randn(hid, k, device="cuda").bfloat16()
        r = torch.randn(m, hid, device="cuda").bfloat16()
        y = torch.empty(m, hid, device="cuda", dtype=torch.bfloat16)
        fl = 2 * m * hid * k
        res[f"{name}_residual"] = fl / _time(lambda: G.gemm(a, w, y, residual=r), iters) / 1e9
        res[f"{name}_plain"] = fl / _time(lambda: G.gemm(a, w, y), iters) / 1e9
        res[f"{name}_cublas"] = fl / _time(lambda: torch.matmul(a, w.t(), out=y), iters) / 1e9
    return res


def gemm_epilogue_profile(epi: str) -> None:
    """Three launches of one fused-epilogue GEMM of the 311M layer (M=8192), for ncu."""
    m, hid, ffn = 8192, 1024, 2736
    x = torch.randn(m, hid, device="cuda").bfloat16()
    if epi == "swiglu":
        w = torch.randn(2 * ffn, hid, device="cuda").bfloat16()
        h = torch.empty(m, ffn, device="cuda", dtype=torch.bfloat16)
        gu = torch.empty(m, 2 * ffn, device="cuda", dtype=torch.bfloat16)
        fn = lambda: G.swiglu_fwd(x, w, ffn, out=h, gate_up=gu)  # noqa: E731
    elif epi == "rope":
        pos = torch.arange(512, device="cuda", dtype=torch.int32)
        inv = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device="cuda").float() / 64))
        w = torch.randn(3 * hid, hid, device="cuda").bfloat16()
        y = torch.empty(m, 3 * hid, device="cuda", dtype=torch.bfloat16)
        fn = lambda: G.qkv_rope_fwd(x, w, pos, inv, 64, 2 * hid, pos_div=m // 512,  # noqa: E731
                                    out=y)
    else:  # residual: the output projection
        w = torch.randn(hid, hid, device="cuda").bfloat16()
        r = torch.randn(m, hid, device="cuda").bfloat16()
        y = torch.empty(m, hid, device="cuda", dtype=torch.bfloat16)
        fn = lambda: G.gemm(x, w, y, residual=r)  # noqa: E731
    for _ in range(3):
        fn()
    torch.cuda.synchronize()


def attn_cases(iters: int) -> dict:
    res = {}
    for b, s, h, hkv, d in [(8, 512, 16, 16, 64), (1, 4096, 8, 2, 128), (1, 8192, 8, 2, 128)]:
        qkv = torch.randn(b, s, h + 2 * hkv, d, device="cuda").bfloat16()
        q, k, v = qkv[:, :, :h], qkv[:, :, h:h + hkv], qkv[:, :, h + hkv:]
        o = torch.empty(b, s, h, d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(b, h, s, device="cuda")
        sc = 1 / math.sqrt(d)
        fl = 4 * b * h * s * s * d / 2
        tag = f"{b}x{s}x{h}/{hkv}x{d}"
        res[f"attn_fwd_{tag}"] = fl / _time(
            lambda: F.flash_fwd(q, k, v, o, lse, sc, True), iters) / 1e9
        res[f"attn_fwd_mma_{tag}"] = fl / _time(
            lambda: lib().flash_attn_fwd(q, k, v, o, lse, sc, True, 0, 0), iters) / 1e9
        dqkv = torch.empty_like(qkv)
        delta = torch.empty(b * h * s, device="cuda")
        acc = torch.empty(b * s * h * d, device="cuda")
        res[f"attn_bwd_{tag}"] = 2.5 * fl / _time(
            lambda: F.attention_bwd(q, k, v, o, o, lse, dqkv[:, :, :h], dqkv[:, :, h:h + hkv],
                                    dqkv[:, :, h + hkv:], causal=True), iters) / 1e9
        res[f"attn_bwd_mma_{tag}"] = 2.5 * fl / _time(
            lambda: lib().flash_attn_bwd(q, k, v, o, o, lse, dqkv[:, :, :h],
                                         dqkv[:, :, h:h + hkv], dqkv[:, :, h + hkv:], delta, acc,
                                         sc, True, 0, 0, None, None, None), iters) / 1e9
        qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))
        res[f"sdpa_fwd_{tag}"] = fl / _time(
            lambda: torch.nn.functional.scaled_dot_product_attention(
                qt, kt, vt, is_causal=True, enable_gqa=True), iters) / 1e9
    return res


def attn_bwd_trace(b: int = 16, s: int = 512, h: int = 16, hkv: int = 16, d: int = 64) -> dict:
    """Phase timing of the tcgen05 attention backward from its in-kernel %globaltimer trace
    (one launch, after warm-up): mean microseconds per CTA phase and per step phase."""
    from ._ext import status_word

    L = lib()
    qkv = torch.randn(b, s, h + 2 * hkv, d, device="cuda").bfloat16()
    q, k, v = qkv[:, :, :h], qkv[:, :, h:h + hkv], qkv[:, :, h + hkv:]
    o = torch.empty(b, s, h, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(b, h, s, device="cuda")
    F.flash_fwd(q, k, v, o, lse, d ** -0.5, True)
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(b * h * s, device="cuda")
    acc = torch.empty(b * s * h * d, device="cuda")
    slots = int(L.attn_bwd_trace_slots())
    ctas = hkv * b * ((s + 127) // 128)
    trace = torch.zeros(ctas * slots, dtype=torch.int64, device="cuda")

    def run(tr):
        L.flash_attn_bwd_prep(o, o, delta, acc)
        L.flash_attn_bwd_tc_kv(q, k, v, o, lse, delta, acc, dqkv[:, :, h:h + hkv],
                               dqkv[:, :, h + hkv:], d ** -0.5, True, 0, 0, None, None,
                               status_word(q.device), trace=tr)
    for _ in range(3):
        run(None)
    run(trace)
    torch.cuda.synchronize()
    t = trace.view(ctas, slots).cpu().double() / 1000.0   # microseconds
    steps = (slots - 3) // 8
    t0 = t[:, 0].min()
    res = {"ctas": ctas, "span_us": float(t[:, 2].max() - t0),
           "cta_us_mean": float((t[:, 2] - t[:, 0]).mean()),
           "setup_us_mean": float((t[:, 1] - t[:, 0]).mean())}
    names = ["sdp_wait", "pds_free_wait", "softmax", "mm_done_wait", "dq_drain"]
    for j, n in enumerate(names):
        col_a, col_b = 3 + j, 4 + j
        vals = []
        for st in range(steps):
            a, bb = t[:, col_a + 6 * st], t[:, col_b + 6 * st]
            ok = (a > 0) & (bb > 0)
            vals.append((bb - a)[ok])
        cat = torch.cat(vals)
        res[f"{n}_us_mean"] = float(cat.mean()) if cat.numel() else None
    gaps = []
    for st in range(steps - 1):
        a, bb = t[:, 3 + 6 * st + 5], t[:, 3 + 6 * (st + 1)]
        ok = (a > 0) & (bb > 0)
        gaps.append((bb - a)[ok])
    cat = torch.cat(gaps)
    res["next_step_gap_us_mean"] = float(cat.mean()) if cat.numel() else None
    last = []
    for i in range(ctas):
        fs = [t[i, 3 + 6 * st + 5] for st in range(steps) if t[i, 3 + 6 * st + 5] > 0]
        if fs:
            last.append(float(t[i, 2] - fs[-1]))
    res["epilogue_us_mean"] = sum(last) / max(1, len(last))
    mq = 3 + 6 * steps
    lag = [(t[:, mq + 2 * st] - t[:, 3 + 6 * st])[(t[:, mq + 2 * st] > 0) & (t[:, 3 + 6 * st] > 0)]
           for st in range(steps)]
    cat = torch.cat(lag)
    res["qdo_landed_minus_step_start_us_mean"] = float(cat.mean()) if cat.numel() else None
    first = t[:, 3]
    res["first_step_start_after_entry_us_mean"] = float((first - t[:, 0])[first > 0].mean())
    ck = 3 + 8 * steps                       # step 0, first chunk: loads, math, stores
    pds0 = t[:, 3 + 2]                       # step 0: P/dS tiles free (chunk loop start)
    for j, n in enumerate(["chunk0_tmem_ld", "chunk0_math", "chunk0_store"]):
        a = pds0 if j == 0 else t[:, ck + j - 1]
        bq = t[:, ck + j]
        ok = (a > 0) & (bq > 0)
        res[f"{n}_us_mean"] = float((bq - a)[ok].mean()) if ok.any() else None
    ok = (t[:, ck + 3] > 0) & (pds0 > 0)
    res["step0_all_chunks_us_mean"] = float((t[:, ck + 3] - pds0)[ok].mean()) if ok.any() else None
    return {k: (round(v, 3) if isinstance(v, float) else v) for k, v in res.items()}


def _hbm_peak_gbs() -> float | None:
    """The measured copy bandwidth of this pool (``MEASURED_PEAKS.json`` at the repo root)."""
    import os

    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def mem_cases(iters: int) -> dict:
    """Memory-bound kernels at 311M-layer widths with 65536 rows (every operand set exceeds
    the 126 MB L2): GB/s of the algorithmic bytes and the fraction of the measured copy
    bandwidth. Bytes count each operand read or written once."""
    rows, h, ffn, heads, d = 65536, 1024, 2736, 16, 64
    dev = "cuda"
    x = torch.randn(rows, h, device=dev).bfloat16()
    w = torch.ones(h, device=dev).bfloat16()
    dy = torch.randn_like(x)
    dres = torch.randn_like(x)
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device=dev)
    dwg = torch.zeros(h, device=dev)
    n = x.numel()
    cases = {
        "rmsnorm_fwd": (4 * n + 4 * rows, lambda: lib().rmsnorm_fwd(x, w, y, rstd, 1e-5)),
        "rmsnorm_bwd_res": (8 * n + 4 * rows,
                            lambda: lib().rmsnorm_bwd(x, w, dy, rstd, y, dwg, dres)),
    }
    gu = torch.randn(rows // 2, 2 * ffn, device=dev).bfloat16()
    dh = torch.randn(rows // 2, ffn, device=dev).bfloat16()
    gout = torch.empty_like(gu)
    cases["swiglu_bwd"] = (10 * (rows // 2) * ffn, lambda: lib().swiglu_bwd(gu, dh, gout))
    b, s = rows // 512, 512
    o = torch.randn(b, s, heads, d, device=dev).bfloat16()
    do = torch.randn_like(o)
    delta = torch.empty(b * heads * s, device=dev)
    dq_acc = torch.empty(o.numel(), device=dev)
    dq = torch.empty_like(o)
    cases["attn_bwd_prep"] = (8 * o.numel() + 4 * delta.numel(),
                              lambda: lib().flash_attn_bwd_prep(o, do, delta, dq_acc))
    cases["attn_dq_convert"] = (6 * o.numel(),
                                lambda: lib().flash_attn_bwd_dq_convert(dq_acc, dq, None, None))
    ids = torch.randint(0, 8192, (rows,), device=dev)
    table = torch.randn(8192, h, device=dev).bfloat16()
    emb = torch.empty(rows, h, device=dev, dtype=torch.bfloat16)
    tgrad = torch.zeros(8192, h, device=dev)
    cases["embedding_fwd"] = (8 * rows + 4 * n, lambda: lib().embedding_fwd(ids, table, 0, emb))
    cases["embedding_bwd"] = (8 * rows + 2 * n + 8 * n,
                              lambda: lib().embedding_bwd(ids, dy, tgrad, 0))
    numel = 80 * 1024 * 1024
    p32 = torch.zeros(numel, device=dev)
    g32 = torch.randn(numel, device=dev)
    m32, v32 = torch.zeros_like(p32), torch.zeros_like(p32)
    plow = torch.empty(numel, device=dev, dtype=torch.bfloat16)
    cases["adamw"] = (30 * numel, lambda: lib().adamw_step(p32, g32, m32, v32, plow, 1e-4, 0.9,
                                                           0.95, 1e-8, 0.1, 1, None, None))
    peak = _hbm_peak_gbs()
    res = {}
    for name, (nbytes, fn) in cases.items():
        gbs = nbytes / _time(fn, iters) / 1e6
        res[f"{name}_GBps"] = gbs
        if peak:
            res[f"{name}_frac_of_measured_hbm"] = gbs / peak
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    if a.case == "gemm_profile":  # a few launches for an ncu capture
        x = torch.randn(4096, 1024, device="cuda").bfloat16()
        w = torch.randn(3072, 1024, device="cuda").bfloat16()
        c = torch.empty(4096, 3072, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            G.gemm(x, w, c)
        torch.cuda.synchronize()
        return
    if a.case.startswith("attn_trace"):   # attn_trace[:d128]
        cfg = (1, 8192, 8, 2, 128) if a.case.endswith("d128") else (16, 512, 16, 16, 64)
        print(json.dumps(attn_bwd_trace(*cfg), indent=1))
        return
    if a.case.startswith("gemm_epi_profile"):  # gemm_epi_profile:swiglu|rope|residual
        gemm_epilogue_profile(a.case.split(":", 1)[1] if ":" in a.case else "swiglu")
        return
    if a.case.startswith("attn_profile"):  # attn_profile[:d128] -> fwd + bwd, 3 launches
        b, s, h, hkv, d = (1, 8192, 8, 2, 128) if a.case.endswith("d128") else (16, 512, 16, 16, 64)
        qkv = torch.randn(b, s, h + 2 * hkv, d, device="cuda").bfloat16()
        q, k, v = qkv[:, :, :h], qkv[:, :, h:h + hkv], qkv[:, :, h + hkv:]
        o = torch.empty(b, s, h, d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(b, h, s, device="cuda")
        dqkv = torch.empty_like(qkv)
        for _ in range(3):
            F.flash_fwd(q, k, v, o, lse, d ** -0.5, True)
            F.attention_bwd(q, k, v, o, o, lse, dqkv[:, :, :h], dqkv[:, :, h:h + hkv],
                            dqkv[:, :, h + hkv:], causal=True)
        torch.cuda.synchronize()
        return
    out = {}
    if a.case in ("all", "gemm"):
        out.update(gemm_cases(a.iters))
    if a.case == "gemm_tiles":
        out.update(gemm_tile_cases(a.iters))
    if a.case in ("all", "gemm_layer"):
        out.update(gemm_layer_cases(a.iters))
    if a.case in ("all", "attn"):
        out.update(attn_cases(a.iters))
    if a.case in ("all", "mem", "norm"):
        out.update(mem_cases(a.iters))
    print(json.dumps({k: round(v, 3 if "frac" in k else 1) for k, v in out.items()}, indent=1))


if __name__ == "__main__":
    main()
