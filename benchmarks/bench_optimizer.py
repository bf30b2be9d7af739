"""Standalone fused AdamW throughput (the expert-parameter update applied in backward).

302M parameters (16 experts x 1536 x 12288, bf16 weights, fp32 gradient) per call, for
both state precisions. Inputs are far larger than L2, so every call streams from HBM.
Reports the CUDA-event time per call and the algorithmic bytes moved per second:

  8bit: grad 4 + weight 2 + m 1 + v 1 + scales 0.25 read, weight 2 + m 1 + v 1 + scales
        0.25 written  = 12.5 B / param
  fp32: grad 4 + weight master 4 + m 4 + v 4 read, master 4 + m 4 + v 4 + bf16 weight 2
        written        = 30 B / param

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
    print(json.dumps(out))


if __name__ == "__main__":
    main()
