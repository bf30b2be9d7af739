"""GEMM and attention throughput on one GPU (reference: benchmark/compute.py).

GEMM [2048, 512] @ [512, 2048] bf16: cuBLAS (torch.mm) vs this framework's tcgen05
GEMM (one group of the grouped kernel). Causal attention [8, 32, 4096, 64] bf16:
torch SDPA with the flash backend. CUDA events, 5 warm-up + 20 timed iterations.

    python benchmarks/compute.py
"""
import json
import os
import sys

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def bench(fn, warmup=5, iters=20):
    torch.cuda.reset_peak_memory_stats()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters, torch.cuda.max_memory_allocated() / 2**20


@torch.inference_mode()
def main():
    from spec_ep.ops.grouped_gemm import gg_fwd

    out = {"gpu": torch.cuda.get_device_name()}
    H, H2 = 2048, 512
    a = torch.randn(H, H2, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(H2, H, device="cuda", dtype=torch.bfloat16)
    c = torch.empty(H, H, device="cuda", dtype=torch.bfloat16)
    flops = 2 * H * H * H2
    ms, mib = bench(lambda: torch.mm(a, b, out=c))
    out["gemm_cublas"] = {"ms": ms, "tflops": flops / ms / 1e9, "peak_mib": mib}
    wt = b.t().contiguous().view(1, H, H2)  # [G=1, N, K]
    off = torch.tensor([0, H], dtype=torch.int32, device="cuda")
    ms, mib = bench(lambda: gg_fwd(a, wt, off, c))
    ref = (a.float() @ b.float())
    out["gemm_tcgen05"] = {"ms": ms, "tflops": flops / ms / 1e9, "peak_mib": mib,
                           "max_rel_err": float((c.float() - ref).abs().max() / ref.abs().max())}
    del a, b, c
    shape = (8, 32, 4096, 64)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    pairs = 4096 * 4097 // 2
    flops = 4 * 8 * 32 * pairs * 64
    with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
        ms, mib = bench(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
    out["attention_sdpa_flash"] = {"ms": ms, "tflops": flops / ms / 1e9, "peak_mib": mib}
    del q, k, v
    out["model_projections"] = model_projections()
    print(json.dumps(out, indent=1))


def model_projections(T=4096):
    """The Qwen3-30B-A3B dense projections at 4096 tokens: forward, input gradient and
    weight gradient on the tcgen05 GEMM (spec_ep.ops.linear) vs cuBLAS (torch.matmul)."""
    from spec_ep.ops.linear import dense_dgrad, dense_fwd, dense_wgrad

    res = {}
    for name, K, N in (("qkv", 2048, 5120), ("o_proj", 4096, 2048), ("router", 2048, 128),
                       ("lm_head", 2048, 151936)):
        x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        gy = torch.randn(T, N, device="cuda", dtype=torch.bfloat16)
        f = 2 * T * K * N
        row = {}
        for op, ours, lib in (("fwd", lambda: dense_fwd(x, w), lambda: x @ w.t()),
                              ("dgrad", lambda: dense_dgrad(gy, w), lambda: gy @ w),
                              ("wgrad", lambda: dense_wgrad(gy, x), lambda: gy.t() @ x)):
            ms, _ = bench(ours)
            ms_lib, _ = bench(lib)
            row[op] = {"ms": ms, "tflops": f / ms / 1e9, "cublas_ms": ms_lib, "cublas_tflops": f / ms_lib / 1e9}
        res[name] = row
        del x, w, gy
    return res


if __name__ == "__main__":
    import argparse

    argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter).parse_args()
    main()
