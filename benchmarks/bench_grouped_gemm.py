"""Time the tcgen05 grouped expert GEMMs against cuBLAS (torch.bmm) on equal shapes.

Shapes default to one Qwen3-30B-A3B MoE layer at EP=8: 16 local experts, 2048 rows per
expert (4096 tokens/rank x top-8 x 8 ranks / 128 experts), hidden 2048, inter 768.

    python benchmarks/bench_grouped_gemm.py [--experts 16 --rows 2048 --hidden 2048 --inter 768]
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def timeit(fn, iters=20, warmup=5, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=768)
    ap.add_argument("--pairs", type=int, default=1, help="256-column tiles on CTA pairs (1) or single CTAs (0)")
    args = ap.parse_args()
    from spec_ep.ops import grouped_gemm as gg
    from spec_ep.ops._ext import load

    load().gemm_set_pairs(bool(args.pairs))

    G, R, H, I = args.experts, args.rows, args.hidden, args.inter
    dev = "cuda"
    x = torch.randn(G * R, H, device=dev).bfloat16()
    wgu = (torch.randn(G, 2 * I, H, device=dev) / H**0.5).bfloat16()
    wd = (torch.randn(G, H, I, device=dev) / I**0.5).bfloat16()
    off = torch.arange(0, G + 1, device=dev, dtype=torch.int32) * R
    flush = torch.empty(256 * 2**20, dtype=torch.int8, device=dev)
    res = {}

    h, gu = gg.gg_swiglu_fwd(x, wgu, off)
    f = 2 * G * R * H * 2 * I
    t = timeit(lambda: gg.gg_swiglu_fwd(x, wgu, off, h, gu), flush=flush)
    tb = timeit(lambda: torch.bmm(x.view(G, R, H), wgu.transpose(1, 2)), flush=flush)
    res["gate_up_swiglu"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    y = gg.gg_fwd(h, wd, off)
    f = 2 * G * R * I * H
    t = timeit(lambda: gg.gg_fwd(h, wd, off, y), flush=flush)
    tb = timeit(lambda: torch.bmm(h.view(G, R, I), wd.transpose(1, 2)), flush=flush)
    res["down"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    dy = torch.randn(G * R, H, device=dev).bfloat16()
    rw = torch.rand(G * R, device=dev)
    dgu, hw, rdw = gg.gg_swiglu_bwd(dy, wd, off, gu, rw)
    f = 2 * G * R * H * I
    t = timeit(lambda: gg.gg_swiglu_bwd(dy, wd, off, gu, rw, dgu, hw, rdw), flush=flush)
    tb = timeit(lambda: torch.bmm(dy.view(G, R, H), wd), flush=flush)
    res["down_dgrad_swiglu_bwd"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    dx = gg.gg_dgrad(dgu, wgu, off)
    f = 2 * G * R * 2 * I * H
    t = timeit(lambda: gg.gg_dgrad(dgu, wgu, off, dx), flush=flush)
    tb = timeit(lambda: torch.bmm(dgu.view(G, R, 2 * I), wgu), flush=flush)
    res["gate_up_dgrad"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    dwgu = gg.gg_wgrad(dgu, x, off, G)
    f = 2 * G * R * 2 * I * H
    t = timeit(lambda: gg.gg_wgrad(dgu, x, off, G, dwgu), flush=flush)
    tb = timeit(lambda: torch.bmm(dgu.view(G, R, 2 * I).transpose(1, 2), x.view(G, R, H)), flush=flush)
    res["gate_up_wgrad"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    dwd = gg.gg_wgrad(dy, hw, off, G)
    f = 2 * G * R * H * I
    t = timeit(lambda: gg.gg_wgrad(dy, hw, off, G, dwd), flush=flush)
    tb = timeit(lambda: torch.bmm(dy.view(G, R, H).transpose(1, 2), hw.view(G, R, I)), flush=flush)
    res["down_wgrad"] = dict(ms=t, tflops=f / t / 1e9, cublas_bmm_ms=tb, cublas_tflops=f / tb / 1e9)

    print(json.dumps({"shape": dict(G=G, rows=R, hidden=H, inter=I), "cta_pairs": bool(args.pairs), "results": res}))


if __name__ == "__main__":
    main()
