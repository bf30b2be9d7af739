"""Small, self-contained cases of the hot kernels for Nsight Compute captures (one GPU).

Each case runs its kernel a few times on inputs larger than L2 (126 MB) but a few GB at
most, so a ``--set full`` capture of one launch ends in seconds:

  gemm      tcgen05 grouped SwiGLU GEMM, 16 experts x 2048 rows, hidden 2048, inter 768
  wgrad     tcgen05 grouped weight gradient (gate_up), same shapes
  dispatch  fused EP receive + combine at world size 1: route plan, count/scan/permute,
            gather of 32,768 expert rows (4096 tokens x top-8, hidden 2048), combine,
            source reduce
  adamw     block-wise 8-bit AdamW on 302M parameters (fp32 gradient)
  attn_fwd / attn_fwd2 / attn_bwd  tcgen05 causal GQA attention (one- and two-tile forward,
            backward), 4096 tokens, 32 query / 4 kv heads
  wgrad_adamw8  expert gate_up weight gradient with the 8-bit AdamW epilogue (128 experts
            x 256 rows, W [128, 1536, 2048])
  layer_ops the model's per-layer elementwise kernels at 16,384 tokens (four sequences'
            worth, above L2): RMSNorm fwd / bwd (hidden 2048), q/k RMSNorm + RoPE fwd / bwd
            (32 / 4 heads), router softmax / top-8 fwd / bwd (128 experts), and the fused
            cross-entropy over a 151,936 vocabulary (4096 tokens)
  dense     the dense projections on the tcgen05 GEMM: QKV forward (4096 x 2048 -> 5120,
            CTA pairs, TMA-store epilogue) and the LM-head input gradient (4096 x 151,936
            -> 2048)
  swiglu_bwd  CTA-pair down-projection dgrad + SwiGLU backward epilogue, 16 experts x 2048
            rows (the EP = 8 layout)

    python benchmarks/ncu_cases.py --case gemm
    ncu --set full --clock-control none -k regex:grouped_gemm -s 2 -c 1 -o out python benchmarks/ncu_cases.py --case gemm
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True, choices=["gemm", "wgrad", "dispatch", "adamw", "wgrad_adamw8", "attn_fwd", "attn_fwd2",
                                                       "attn_bwd", "layer_ops", "dense", "swiglu_bwd"])
    ap.add_argument("--reps", type=int, default=4)
    args = ap.parse_args()
    from spec_ep.ops import grouped_gemm as gg

    torch.manual_seed(0)
    dev = "cuda"
    if args.case in ("gemm", "wgrad"):
        G, R, H, I = 16, 2048, 2048, 768
        x = torch.randn(G * R, H, device=dev).bfloat16()
        w = (torch.randn(G, 2 * I, H, device=dev) / H**0.5).bfloat16()
        off = torch.arange(0, G + 1, device=dev, dtype=torch.int32) * R
        h, gu = gg.gg_swiglu_fwd(x, w, off)
        out = torch.empty(G, 2 * I, H, device=dev)
        for _ in range(args.reps):
            if args.case == "gemm":
                gg.gg_swiglu_fwd(x, w, off, h, gu)
            else:
                gg.gg_wgrad(gu, x, off, G, out)
    elif args.case == "dispatch":
        from spec_ep.parallel.ep import ExpertParallel
        from spec_ep.utils.routing import synthetic_routing

        ep = ExpertParallel(128, 8, 2048, max_tokens=4096)
        x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, device=dev)
        for _ in range(args.reps):
            st = ep.dispatch_fwd(x, te, tw)
            ep.combine_fwd(st.xp, st)
        ep.check()
    elif args.case in ("attn_fwd", "attn_fwd2", "attn_bwd"):
        from spec_ep.ops.attention import attention_bwd, attention_fwd

        T, Hq, Hkv = 4096, 32, 4
        q = torch.randn(T, Hq, 128, device=dev).bfloat16()
        k = torch.randn(T, Hkv, 128, device=dev).bfloat16()
        v = torch.randn(T, Hkv, 128, device=dev).bfloat16()
        do = torch.randn(T, Hq * 128, device=dev).bfloat16()
        o, lse = attention_fwd(q, k, v)
        for _ in range(args.reps):
            if args.case in ("attn_fwd", "attn_fwd2"):
                attention_fwd(q, k, v, two_tile=args.case == "attn_fwd2")
            else:
                attention_bwd(q, k, v, o, lse, do)
    elif args.case == "layer_ops":
        from spec_ep.ops._ext import load

        C = load()
        T, H = 16384, 2048
        x = torch.randn(T, H, device=dev).bfloat16()
        w = torch.ones(H, device=dev).bfloat16()
        y = torch.empty_like(x)
        rstd = torch.empty(T, device=dev)
        dx = torch.empty_like(x)
        dw = torch.zeros(H, device=dev)
        qkv = torch.randn(T, 40 * 128, device=dev).bfloat16()
        logits = torch.randn(T, 128, device=dev)
        te = torch.empty(T, 8, device=dev, dtype=torch.int32)
        tw = torch.empty(T, 8, device=dev)
        probs = torch.empty(T, 128, device=dev)
        from spec_ep.ops.rope import qk_norm_rope

        wq = torch.ones(128, device=dev).bfloat16().requires_grad_()
        wk = torch.ones(128, device=dev).bfloat16().requires_grad_()
        lg = torch.randn(4096, 151936, device=dev).bfloat16()
        labels = torch.randint(0, 151936, (4096,), device=dev).int()
        loss = torch.empty(4096, device=dev)
        for _ in range(args.reps):
            C.rmsnorm_fwd(x, w, y, rstd, 1e-6, None, None)
            C.rmsnorm_bwd(x, w, rstd, y, dx, dw, None)
            q, kk, v = qk_norm_rope(qkv.requires_grad_(), wq, wk, 32, 4)
            torch.autograd.backward([q, kk, v], [torch.ones_like(q), torch.ones_like(kk), torch.ones_like(v)])
            C.router_topk(logits, None, 8, True, te, tw, probs)
            C.router_bwd(probs, te, tw, True, logits)
            C.xent_fwd_bwd(lg, labels, 1.0 / 4096, loss)
    elif args.case == "dense":
        from spec_ep.ops.linear import dense_dgrad, dense_fwd

        x = torch.randn(4096, 2048, device=dev).bfloat16()
        wqkv = (torch.randn(5120, 2048, device=dev) * 0.02).bfloat16()
        gy = torch.randn(4096, 151936, device=dev).bfloat16()
        wlm = (torch.randn(151936, 2048, device=dev) * 0.02).bfloat16()
        for _ in range(args.reps):
            dense_fwd(x, wqkv)
            dense_dgrad(gy, wlm)
    elif args.case == "swiglu_bwd":
        G, R, H, I = 16, 2048, 2048, 768
        dy = torch.randn(G * R, H, device=dev).bfloat16()
        wd = (torch.randn(G, H, I, device=dev) / H**0.5).bfloat16()
        gu = torch.randn(G * R, 2 * I, device=dev).bfloat16()
        rw = torch.rand(G * R, device=dev)
        off = torch.arange(0, G + 1, device=dev, dtype=torch.int32) * R
        for _ in range(args.reps):
            gg.gg_swiglu_bwd(dy, wd, off, gu, rw)
    elif args.case == "wgrad_adamw8":
        from spec_ep.ops.optim import FusedAdamW

        G, rows, M, N = 128, 256, 1536, 2048
        a = (torch.randn(G * rows, M, device=dev) * 0.1).bfloat16()
        b = (torch.randn(G * rows, N, device=dev) * 0.1).bfloat16()
        off = torch.arange(0, G + 1, device=dev, dtype=torch.int32) * rows
        p = torch.nn.Parameter((torch.randn(G, M, N, device=dev) * 0.02).bfloat16())
        p._sepx_state_precision = "8bit"
        opt = FusedAdamW([p], lr=1e-4)
        for _ in range(args.reps):
            opt.fused_wgrad(p, a, b, off)
    else:
        from spec_ep.ops.optim import FusedAdamW

        p = torch.nn.Parameter((torch.randn(16, 1536, 2048 * 6, device=dev) * 0.02).bfloat16())
        p._sepx_state_precision = "8bit"
        opt = FusedAdamW([p], lr=1e-4)
        g = torch.randn(p.shape, device=dev) * 1e-3
        for _ in range(args.reps):
            opt.apply_now(p, g)
    torch.cuda.synchronize()
    print(f"case {args.case} ok")


if __name__ == "__main__":
    main()
