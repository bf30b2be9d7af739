"""Standalone fused AdamW throughput (the expert-parameter update applied in backward).

302M parameters (16 experts x 1536 x 12288, bf16 weights, fp32 gradient) per call, for
both state precisions. Inputs are far larger than L2, so every call streams from HBM.
Reports the CUDA-event time per call and the algorithmic bytes moved per second:

  8bit: grad 4 + weight 2 + m 1 + v 1 + scales 0.25 read, weight 2 + m 1 + v 1 + scales
        0.25 written  = 12.5 B / param
  fp32: grad 4 + weight master 4 + m 4 + v 4 read, master 4 + m 4 + v 4 + bf16 weight 2
        written        = 30 B / param

Then the expert weight update as training runs it on one GPU (Qwen3-30B-A3B, 128
experts, 256 tokens each = 32768 routed rows): weight-gradient GEMM to an fp32 gradient
followed by the streaming optimizer, vs the GEMM whose epilogue applies 8-bit AdamW.

    python benchmarks/bench_optimizer.py
"""
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

BYTES = {"8bit": 12.5, "fp32": 30.0}


def main():
    from spec_ep.ops.optim import FusedAdamW

    out = {}
    for prec in ("8bit", "fp32"):
        p = torch.nn.Parameter((torch.randn(16, 1536, 2048 * 6, device="cuda") * 0.02).bfloat16())
        p._sepx_state_precision = prec
        opt = FusedAdamW([p], lr=1e-4)
        g = torch.randn(p.shape, device="cuda") * 1e-3
        for _ in range(3):
            opt.apply_now(p, g)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iters = 10
        s.record()
        for _ in range(iters):
            opt.apply_now(p, g)
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / iters
        n = p.numel()
        out[prec] = {"params": n, "ms_per_call": ms, "algorithmic_GBps": BYTES[prec] * n / ms / 1e6}
        del p, opt, g
        torch.cuda.empty_cache()

    from spec_ep.ops.grouped_gemm import gg_wgrad

    G, rows = 128, 256
    go = torch.arange(0, G + 1, device="cuda", dtype=torch.int32) * rows
    for name, M, N in (("gate_up", 1536, 2048), ("down", 2048, 768)):
        a = (torch.randn(G * rows, M, device="cuda") * 0.1).bfloat16()
        b = (torch.randn(G * rows, N, device="cuda") * 0.1).bfloat16()
        p = torch.nn.Parameter((torch.randn(G, M, N, device="cuda") * 0.02).bfloat16())
        p._sepx_state_precision = "8bit"
        opt = FusedAdamW([p], lr=1e-4)
        grad = torch.empty(G, M, N, device="cuda")

        def unfused():
            gg_wgrad(a, b, go, G, out=grad)
            opt.apply_now(p, grad)

        def fused():
            opt.fused_wgrad(p, a, b, go)

        row = {"shape": [G, M, N], "rows_per_expert": rows}
        for label, fn in (("unfused_ms", unfused), ("fused_ms", fused)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(10):
                fn()
            e.record()
            e.synchronize()
            row[label] = s.elapsed_time(e) / 10
        row["fused_state_GBps"] = 8.5 * p.numel() / row["fused_ms"] / 1e6
        out["wgrad_" + name] = row
        del a, b, p, opt, grad
        torch.cuda.empty_cache()
    print(json.dumps(out))


if __name__ == "__main__":
    import argparse

    argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter).parse_args()
    main()
