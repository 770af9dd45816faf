"""Kernel microbenchmarks: CUDA-event timing of each sm_100a kernel vs its library baseline.

    python -m nano_megatron_b200.ops.bench_kernels [--case all|gemm|attn|norm] [--iters N]

Prints one JSON object of achieved TFLOP/s (GEMM, attention) or GB/s (memory-bound
kernels). Also the small, self-contained workload used for ncu captures
(``--case gemm_profile`` / ``attn_profile`` run a few launches of one kernel).
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


def norm_cases(iters: int) -> dict:
    x = torch.randn(32768, 1024, device="cuda").bfloat16()
    w = torch.ones(1024, device="cuda").bfloat16()
    y = torch.empty_like(x)
    r = torch.empty(32768, device="cuda")
    nbytes = 2 * x.numel() * 2
    return {"rmsnorm_fwd_GBps": nbytes / _time(lambda: lib().rmsnorm_fwd(x, w, y, r, 1e-5),
                                               iters) / 1e6}


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
    if a.case == "attn_profile":
        b, s, h, d = 8, 512, 16, 64
        qkv = torch.randn(b, s, 3 * h, d, device="cuda").bfloat16()
        o = torch.empty(b, s, h, d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(b, h, s, device="cuda")
        for _ in range(3):
            F.flash_fwd(qkv[:, :, :h], qkv[:, :, h:2 * h], qkv[:, :, 2 * h:], o, lse, 0.125, True)
        torch.cuda.synchronize()
        return
    out = {}
    if a.case in ("all", "gemm"):
        out.update(gemm_cases(a.iters))
    if a.case in ("all", "attn"):
        out.update(attn_cases(a.iters))
    if a.case in ("all", "norm"):
        out.update(norm_cases(a.iters))
    print(json.dumps({k: round(v, 1) for k, v in out.items()}, indent=1))


if __name__ == "__main__":
    main()
