"""Even vs uneven (real-routing) token all-to-all (reference: benchmark/all2all/even_vs_uneven.py).

Per-rank routing comes from ``experts_rank{r}.pt`` dumps ([L, T, K]) when ``--run-dir``
is given, else from synthetic Zipf routing. Times, for the uneven (routing) and even
splits: NCCL ``all_to_all_single`` of bf16 rows (one row per (token, expert), the
reference's scheme) and this framework's P2P dispatch + combine (one row per (token,
rank)). Max over ranks of CUDA-event time.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/all2all_even_vs_uneven.py [--run-dir logs/x --layer 0]
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def timed(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--run-dir", default=None)
    ap.add_argument("--layer", type=int, default=0)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--zipf", type=float, default=1.0)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.utils.dist import init_distributed
    from spec_ep.utils.routing import synthetic_routing

    rank, world, dev = init_distributed()
    E, H = args.experts, args.hidden
    if args.run_dir:
        ids = torch.load(f"{args.run_dir}/experts_rank{rank}.pt")[args.layer].long()
        x = torch.randn(ids.shape[0], H, device=dev).bfloat16()
        te = ids.int().to(dev)
        tw = torch.full(te.shape, 1.0 / te.shape[1], device=dev)
    else:
        x, te, tw = synthetic_routing(args.tokens, H, E, args.top_k, s=args.zipf, rank=rank, device=dev)
    T, k = te.shape
    send = torch.bincount(te.long().flatten() // (E // world), minlength=world)
    counts = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(counts, send)
    counts = torch.stack(counts).cpu()
    s_spl, r_spl = counts[rank].tolist(), counts[:, rank].tolist()
    res = {"world": world, "tokens": T, "top_k": k, "hidden": H}
    rows = torch.randn(sum(s_spl), H, device=dev).bfloat16()
    out = torch.empty(sum(r_spl), H, device=dev).bfloat16()
    res["nccl_uneven_ms"] = timed(lambda: dist.all_to_all_single(out, rows, r_spl, s_spl), args.iters)
    even = [T * k // world] * world
    rows_e = torch.randn(sum(even), H, device=dev).bfloat16()
    out_e = torch.empty_like(rows_e)
    res["nccl_even_ms"] = timed(lambda: dist.all_to_all_single(out_e, rows_e, even, even), args.iters)
    off_rank = (sum(s_spl) - s_spl[rank]) * H * 2
    res["nccl_uneven_offrank_MiB"] = off_rank / 2**20
    ep = ExpertParallel(E, k, H, max_tokens=T, device=dev)

    def p2p():
        st = ep.dispatch_fwd(x, te, tw)
        ep.combine_fwd(st.xp, st)

    res["p2p_dispatch_combine_ms"] = timed(p2p, args.iters)
    ep.check()
    if rank == 0:
        print(json.dumps(res), flush=True)
    ep.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
