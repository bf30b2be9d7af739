"""MoE-layer dispatch + combine benchmarks (identity experts, so only data movement counts).

Scenarios (all on synthetic routing: x ~ N(0,1), router W ~ N(0, 0.02) plus a per-expert
Zipf bias of exponent s; max over ranks of CUDA-event time):

  layer    Qwen3-30B-A3B MoE layer: hidden 2048, 128 experts, top-8, 4096 tokens/rank,
           Zipf s=1.0, seeds 0-4. Fused P2P path vs naive per-copy NCCL all-to-all vs
           the reference's RBD_combine_dispatch (unmodified, when installed).
  fp8      inference dispatch with e4m3 1x128 payload: prefill 8192 and decode 128
           tokens/rank, Zipf s=1.0, with and without replicating the 16 hottest experts
           on every rank.
  graph    decode: 128 tokens/rank, fp8 payload, 16 hottest experts replicated, identity
           experts; eager layers vs the same 8 layers replayed from one CUDA graph
           (device-side epochs, no host sync), time per layer.
  hier     Qwen3-235B-A22B MoE layer (hidden 4096, 128 experts, top-8, 4096 tokens/rank)
           on logical groups of --group-size: two-stage path vs flat P2P vs naive NCCL,
           Zipf s in {0, 0.5, 1.0, 1.5}.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/bench_dispatch.py --scenario layer fp8 hier
"""
import argparse
import importlib.util
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def timed(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters * 1000.0], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def reference_rbd():
    path = os.path.join(ROOT, "baseline", "_ref", "spec_ep", "rbd.py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("reference_spec_ep_rbd", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def rows_per_token(te, e2r, rank, world):
    dst = e2r[te.long()]
    T = te.shape[0]
    naive = float((dst != rank).sum()) / T
    hot = torch.zeros(T, world, dtype=torch.bool, device=te.device)
    hot.scatter_(1, dst.long(), True)
    dedup = float(hot.sum() - hot[:, rank].sum()) / T
    return naive, dedup


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--scenario", nargs="+", default=["layer", "fp8", "graph", "hier"])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--group-size", type=int, default=4)
    ap.add_argument("--profile", action="store_true",
                    help="per-kernel device times of the fused layer path (torch profiler, every rank)")
    args = ap.parse_args()
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.parallel.hierarchical import HierarchicalEP
    from spec_ep.parallel.placement import plan_balanced
    from spec_ep.rbd import naive_combine_dispatch
    from spec_ep.utils.dist import init_distributed
    from spec_ep.utils.routing import synthetic_routing

    rank, world, dev = init_distributed()
    if not dist.is_initialized():  # a single rank still uses the collectives below
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29560")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
    out = {"world": world}
    ident = lambda rows, ids: rows  # noqa: E731
    ref = reference_rbd()
    local_group, _ = dist.new_subgroups(group_size=world)

    if "layer" in args.scenario:
        ep = ExpertParallel(128, 8, 2048, max_tokens=4096, device=dev)
        res = []
        for seed in range(5):
            x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=seed, rank=rank, device=dev)

            def p2p():  # one layer per pass: the training step's row budget, no host wait
                ep.begin_pass()
                st = ep.dispatch_fwd(x, te, tw)
                ep.combine_fwd(st.xp, st)

            p2p()
            ep.end_pass()  # learn the row budget (exact sizes once)
            r = {"seed": seed, "p2p_us": timed(p2p, args.iters)}
            assert not ep.end_pass(), "row budget outgrown inside the timed loop"
            if seed == 0:
                # host cost of issuing one layer call (no sync inside the loop): when it
                # approaches p2p_us the layer is bound by the host, not the GPU
                import time

                torch.cuda.synchronize()
                dist.barrier()
                t0 = time.perf_counter()
                for _ in range(args.iters):
                    p2p()
                r["host_issue_us"] = (time.perf_counter() - t0) * 1e6 / args.iters
                torch.cuda.synchronize()
                ep.end_pass()
                r["host_cpus"] = os.cpu_count()
            r["nccl_naive_us"] = timed(lambda: naive_combine_dispatch(x, tw, ident, te.long(), 128), args.iters)
            if ref is not None:
                r["reference_rbd_us"] = timed(lambda: ref.RBD_combine_dispatch(
                    x, tw, ident, te.long(), E=128, gpus_per_node=world, local_group=local_group, concurrent=True),
                    args.iters)
            r["naive_rows_per_token"], r["dedup_rows_per_token"] = rows_per_token(te, ep.e2r, rank, world)
            res.append(r)
        ep.check()
        ep.close()
        out["layer"] = res

    if args.profile:
        from torch.profiler import ProfilerActivity, profile

        ep = ExpertParallel(128, 8, 2048, max_tokens=4096, device=dev)
        x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=0, rank=rank, device=dev)

        def p2p():
            ep.begin_pass()
            st = ep.dispatch_fwd(x, te, tw)
            ep.combine_fwd(st.xp, st)

        for _ in range(3):
            p2p()
        ep.end_pass()
        torch.cuda.synchronize()
        dist.barrier()
        with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
            for _ in range(5):
                p2p()
            torch.cuda.synchronize()
        ep.check()
        ep.close()
        if rank in (0, world - 1):
            print(f"--- rank {rank} ---")
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=18), flush=True)
        dist.barrier()

    if "fp8" in args.scenario:
        res = []
        for T in (8192, 128):
            for rep in (0, 16):
                x, te, tw = synthetic_routing(T, 2048, 128, 8, s=1.0, seed=0, rank=rank, device=dev)
                load = torch.bincount(te.flatten().long(), minlength=128).float()
                dist.all_reduce(load)
                placement = plan_balanced(load.cpu(), world, replicate_top=rep) if rep else None
                row = {"tokens": T, "replicate_top": rep}
                for fp8 in (False, True):
                    ep = ExpertParallel(128, 8, 2048, max_tokens=T, device=dev, fp8_dispatch=fp8, placement=placement)

                    def p2p():
                        ep.begin_pass()
                        st = ep.dispatch_fwd(x, te, tw)
                        ep.combine_fwd(st.xp, st)

                    p2p()
                    ep.end_pass()
                    row["fp8_us" if fp8 else "bf16_us"] = timed(p2p, args.iters)
                    assert not ep.end_pass(), "row budget outgrown inside the timed loop"
                    ep.check()
                    row["dedup_rows_per_token"] = rows_per_token(te, ep.e2r, rank, world)[1]
                    ep.close()
                row["bytes_per_row"] = {"bf16": 2048 * 2, "fp8": 2048 + 16 * 4}
                res.append(row)
        out["fp8"] = res

    if "graph" in args.scenario:
        from spec_ep.parallel.ep import EPGraph

        T, L = 128, 8
        res = []
        for fp8 in (False, True):
            x, te, tw = synthetic_routing(T, 2048, 128, 8, s=1.0, seed=0, rank=rank, device=dev)
            load = torch.bincount(te.flatten().long(), minlength=128).float()
            dist.all_reduce(load)
            placement = plan_balanced(load.cpu(), world, replicate_top=16)
            ep = ExpertParallel(128, 8, 2048, max_tokens=T, device=dev, fp8_dispatch=fp8, placement=placement)

            def layers(static):
                y = x
                for _ in range(L):
                    st = ep.dispatch_fwd(y, te, tw, static_rows=static)
                    y = ep.combine_fwd(st.xp, st)
                return y

            row = {"tokens": T, "fp8": fp8, "replicate_top": 16}
            row["eager_us_per_layer"] = timed(lambda: layers(False), args.iters) / L
            g = EPGraph(ep, lambda: layers(True))
            row["graph_us_per_layer"] = timed(g.replay, args.iters) / L
            ep.check()
            del g
            ep.graph_epochs(False)
            ep.close()
            res.append(row)
        out["graph"] = res

    if "hier" in args.scenario and world % args.group_size == 0:
        res = []
        T, H = 4096, 4096
        hep = HierarchicalEP(128, 8, H, max_tokens=T, group_size=args.group_size, device=dev)
        ep = ExpertParallel(128, 8, H, max_tokens=T, device=dev)
        for s in (0.0, 0.5, 1.0, 1.5):
            x, te, tw = synthetic_routing(T, H, 128, 8, s=s, seed=0, rank=rank, device=dev)
            row = {"zipf": s}
            row["hier_us"] = timed(lambda: hep.forward(x, te, tw), args.iters)
            hep.check()
            row["pilot_rows_per_token"] = float(hep.last_pilot_rows.sum()) / T

            def flat():
                st = ep.dispatch_fwd(x, te, tw)
                ep.combine_fwd(st.xp, st)

            row["flat_p2p_us"] = timed(flat, args.iters)
            row["nccl_naive_us"] = timed(lambda: naive_combine_dispatch(x, tw, ident, te.long(), 128), args.iters)
            row["naive_rows_per_token"], row["dedup_rows_per_token"] = rows_per_token(te, ep.e2r, rank, world)
            res.append(row)
        ep.check()
        hep.close()
        ep.close()
        out["hier"] = {"group_size": args.group_size, "rows": res}

    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
