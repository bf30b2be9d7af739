"""Replay recorded routing through placements and the speculative replica cache (CPU).

Input: one ``experts_rank{r}.pt`` dump per source rank (int16 ``[L, T, K]``, written by
``spec_ep.utils.profile.RoutingRecorder`` / ``examples/ds_moe.py --modes routing``), or
``--synthetic`` Zipf-routed dumps. Per layer, prints one JSON line per scheme:

  contiguous         experts e // (E / world) (the reference's layout)
  balanced           LPT packing of the dump's loads
  replicate_top{n}   balanced + the n hottest experts on every rank
  copies{c}          balanced + the n hottest experts on c ranks each
  cache{S}_{pred}    contiguous + each rank's LRU replica cache of S slots, predicted
                     from the step's own routing (oracle) or the previous step's

with remote rows per token (per-rank dedup) against the naive per-copy count, the
receive imbalance, the worst rank's max(sent, received) rows per token (what bounds the
dispatch's link time), and for the caches hits, fetches, the expert weight bytes fetched
and the token bytes kept off NVLink (dispatch rows + combine partials) against the
contiguous layout: the cache pays where the second exceeds the first.

    python benchmarks/replay_routing.py logs/run/experts_rank*.pt --world 8 --tokens-per-step 128
    python benchmarks/replay_routing.py --synthetic --world 8 --num-experts 128 --top-k 8
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("files", nargs="*")
    ap.add_argument("--world", type=int, default=None, help="EP ranks (default: number of files)")
    ap.add_argument("--num-experts", type=int, default=128)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--layers", type=int, nargs="*", default=None)
    ap.add_argument("--replicate-top", type=int, default=16)
    ap.add_argument("--copies", type=int, default=2)
    ap.add_argument("--slots", type=int, default=16)
    ap.add_argument("--tokens-per-step", type=int, default=128)
    ap.add_argument("--min-count", type=int, default=1, help="cache experts predicted for >= this many tokens")
    ap.add_argument("--interval", type=int, default=1, help="re-plan the caches every this many steps")
    ap.add_argument("--expert-bytes", type=int, default=3 * 2048 * 768 * 2)
    ap.add_argument("--row-bytes", type=int, default=2048 * 2, help="bytes of one token row (bf16 hidden)")
    ap.add_argument("--synthetic", action="store_true", help="Zipf-routed dumps instead of files")
    ap.add_argument("--zipf", type=float, default=1.0)
    ap.add_argument("--tokens", type=int, default=1024, help="tokens per rank of a synthetic dump")
    ap.add_argument("--drift-every", type=int, default=0,
                    help="synthetic: re-draw which experts are hot every this many steps (0: stationary); "
                         "static placements are then planned from the first step only")
    ap.add_argument("--hidden", type=int, default=2048,
                    help="hidden size of a synthetic dump's router (the logit spread grows with it, so it sets "
                         "how much the Zipf bias dominates; 2048 is the dispatch benchmarks' layer)")
    args = ap.parse_args(argv)
    from spec_ep.parallel.placement import contiguous, plan_balanced
    from spec_ep.parallel.simulate import placement_traffic, replay_cache, split_steps
    from spec_ep.utils.routing import synthetic_routing

    if args.synthetic:
        W = args.world or 8
        dumps = []
        for r in range(W):
            if args.drift_every:
                n_steps = max(args.tokens // args.tokens_per_step, 1)
                parts = [synthetic_routing(args.tokens_per_step, args.hidden, args.num_experts, args.top_k,
                                           s=args.zipf, seed=0, rank=r, bias_seed=i // args.drift_every,
                                           token_seed=i)[1] for i in range(n_steps)]
                te = torch.cat(parts)
            else:
                _, te, _ = synthetic_routing(args.tokens, args.hidden, args.num_experts, args.top_k, s=args.zipf,
                                             seed=0, rank=r)
            dumps.append(te.long().unsqueeze(0))
    else:
        if not args.files:
            ap.error("give dump files or --synthetic")
        dumps = [torch.load(f).long() for f in args.files]
        W = args.world or len(dumps)
        if len(dumps) != W:
            ap.error(f"{len(dumps)} dump files for {W} ranks: give one file per source rank")
    E = args.num_experts
    L = dumps[0].shape[0]
    out = []
    for l in (args.layers if args.layers is not None else range(L)):
        routes = [d[l] for d in dumps]
        seen = [r[:args.tokens_per_step] for r in routes] if args.drift_every else routes  # what the planner knows
        load = torch.bincount(torch.cat(seen).reshape(-1), minlength=E).float()
        schemes = {"contiguous": contiguous(E, W), "balanced": plan_balanced(load, W),
                   f"replicate_top{args.replicate_top}": plan_balanced(load, W, args.replicate_top)}
        if 1 < args.copies < W:
            schemes[f"copies{args.copies}_top{args.replicate_top}"] = plan_balanced(load, W, args.replicate_top,
                                                                                    args.copies)
        for name, pl in schemes.items():
            rec = {"layer": l, "scheme": name, **placement_traffic(routes, pl)}
            rec.pop("recv_rows")
            out.append(rec)
        steps = split_steps(dumps, l, args.tokens_per_step)
        for pred in ("oracle", "previous"):
            res = replay_cache(steps, contiguous(E, W), args.slots, predict=pred, expert_bytes=args.expert_bytes,
                               row_bytes=args.row_bytes, min_count=args.min_count, interval=args.interval)
            out.append({"layer": l, "scheme": f"cache{args.slots}_{pred}", "steps": len(steps),
                        "remote_rows_per_token": res["mean_remote_rows_per_token"],
                        "naive_rows_per_token": sum(s["naive_rows_per_token"] for s in res["steps"]) / len(steps),
                        "recv_imbalance": res["mean_recv_imbalance"],
                        "worst_link_rows_per_token": sum(s["worst_link_rows_per_token"] for s in res["steps"])
                        / len(steps), "hits": res["hits"],
                        "fetches": res["fetches"], "hit_rate": res["hit_rate"],
                        "fetched_MiB": res["fetched_bytes"] / 2**20,
                        "token_MiB_saved": res["saved_bytes"] / 2**20})
    for rec in out:
        print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in rec.items()}))
    return out


if __name__ == "__main__":
    main()
