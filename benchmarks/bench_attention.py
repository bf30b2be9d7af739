"""Causal GQA attention: tcgen05 kernels vs torch SDPA (cuDNN / flash backend).

Qwen3-30B-A3B attention shape by default: 4096 tokens, 32 query heads, 4 kv heads,
head_dim 128, bf16. Forward and backward, CUDA-event timed after 3 warm-up calls. The
inputs (≈ 50 MB) stay L2-resident between iterations, as they do inside a training step
where attention re-reads K/V from L2 by design. FLOPs count the causal half only
(backward = 2.5 x forward).

    python benchmarks/bench_attention.py [--T 4096 --hq 32 --hkv 4]
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def timed(fn, iters=20, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    from spec_ep.ops.attention import attention_bwd, attention_fwd, causal_gqa_attention

    T, Hq, Hkv = args.T, args.hq, args.hkv
    torch.manual_seed(0)
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    do = torch.randn(T, Hq * 128, device="cuda").bfloat16()
    fwd_flops = 4 * Hq * (T * (T + 1) // 2) * 128
    bwd_flops = 2.5 * fwd_flops

    o, lse = attention_fwd(q, k, v)
    out = {"T": T, "Hq": Hq, "Hkv": Hkv}
    out["tc_fwd_us"] = timed(lambda: attention_fwd(q, k, v), args.iters)
    out["tc2_fwd_us"] = timed(lambda: attention_fwd(q, k, v, two_tile=True), args.iters)
    o2, _ = attention_fwd(q, k, v, two_tile=True)
    out["tc2_fwd_maxdiff_vs_tc"] = (o2.float() - o.float()).abs().max().item()
    out["tc_bwd_us"] = timed(lambda: attention_bwd(q, k, v, o, lse, do), args.iters)

    qs, ks, vs = (t.clone().requires_grad_() for t in (q, k, v))
    out["sdpa_fwd_us"] = timed(lambda: causal_gqa_attention(qs, ks, vs), args.iters)
    os_ = causal_gqa_attention(qs, ks, vs)
    out["sdpa_bwd_us"] = timed(lambda: torch.autograd.grad(os_, (qs, ks, vs), do, retain_graph=True), args.iters)
    out["tc2_fwd_tflops"] = fwd_flops / out["tc2_fwd_us"] / 1e6
    for name in ("tc", "sdpa"):
        out[f"{name}_fwd_tflops"] = fwd_flops / out[f"{name}_fwd_us"] / 1e6
        out[f"{name}_bwd_tflops"] = bwd_flops / out[f"{name}_bwd_us"] / 1e6
    out["fwd_maxdiff"] = (o.float() - os_.float()).abs().max().item()
    dq, dk, dv = attention_bwd(q, k, v, o, lse, do)
    gq, gk, gv = torch.autograd.grad(os_, (qs, ks, vs), do)
    out["bwd_rel"] = [((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
                      for a, b in ((dq, gq), (dk, gk), (dv, gv))]
    print(json.dumps(out))


if __name__ == "__main__":
    main()
