"""Speculative expert replication benchmark (inference, Qwen3-30B-A3B-shaped layers).

A ``--layers``-deep Qwen3-30B-A3B-shaped decoder (hidden 2048, 32 / 4 heads, 128 experts,
top-8, inter 768; random init) with a per-expert Zipf router bias of exponent ``--zipf``
(a different hot set per layer). Two cases per rank and call: ``prefill`` (8192 tokens
per rank, one call) and ``decode`` (128 tokens per rank, repeated calls with new tokens).
Each runs without speculation, then with an LRU replica cache of ``--slots`` experts per
layer and rank (prediction: the layer's router on the incoming residual stream; fetch
overlapped with attention). Reports device time per layer (CUDA events, max over ranks),
remote rows per token (one row per (token, other rank)), the share of the tokens'
non-local choices that the cache served locally, and cache hits / fetches.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/bench_speculative.py
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--slots", type=int, default=16)
    ap.add_argument("--zipf", type=float, default=1.0)
    ap.add_argument("--fp8", action="store_true", help="e4m3 1x128 dispatch payload")
    ap.add_argument("--cases", nargs="+", default=["prefill", "decode"])
    ap.add_argument("--decode-steps", type=int, default=20)
    ap.add_argument("--predictor", choices=["router", "mlp"], default="router")
    ap.add_argument("--interval", type=int, default=1, help="re-plan the caches every N calls")
    args = ap.parse_args()

    from spec_ep.models.config import get_config
    from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.parallel.speculative import enable_speculation
    from spec_ep.utils.dist import init_distributed
    from spec_ep.utils.routing import zipf_bias

    rank, world, dev = init_distributed("nccl", timeout_s=300)
    multi = dist.is_initialized()

    def all_reduce(t, op=dist.ReduceOp.SUM):
        if multi:
            dist.all_reduce(t, op=op)

    def barrier():
        if multi:
            dist.barrier()
    cfg = get_config("qwen3-30b-a3b", num_layers=args.layers)
    E = cfg.num_experts

    def build(T):
        ep = ExpertParallel(E, cfg.top_k, cfg.hidden_size, max_tokens=T, device=dev, fp8_dispatch=args.fp8)
        torch.manual_seed(0)
        model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
        model.eval()
        for l, layer in enumerate(model.layers):
            # Zipf popularity in logit space, as the dispatch benchmarks' synthetic routing
            layer.router_logit_bias = zipf_bias(E, args.zipf, seed=l, device=dev)
        return ep, model

    def run_case(name, T, calls):
        ep, model = build(T)
        captured = []
        for l, layer in enumerate(model.layers):
            layer.routing_callback = (lambda te, l=l: captured.append((l, te.clone())))
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        batches = [torch.randint(0, cfg.vocab_size, (1, T), device=dev, generator=g) for _ in range(calls)]

        def go(warm):  # one pass per call: no host read between the layers
            for ids in (batches[:warm] if warm else batches):
                ep.run_pass(lambda: model.hidden_states(ids.view(-1)))

        def measure(label):
            # untimed pass over every batch: warms kernels and, with speculation, the caches
            captured.clear()
            go(0)
            torch.cuda.synchronize()
            rows = []
            local, remote = 0, 0
            for l, te in captured[-args.layers:]:
                layer = model.layers[l]
                e2r = layer.spec.cache.e2r if layer.spec is not None else ep.e2r
                base = ep.e2r if layer.spec is None else layer.spec.cache.base_e2r
                dst = e2r[te.long()]
                hot = torch.zeros(te.shape[0], world, dtype=torch.bool, device=dev).scatter_(1, dst.long(), True)
                rows.append(float(hot.sum() - hot[:, rank].sum()) / te.shape[0])
                far = base[te.long()] != rank
                remote += int(far.sum())
                local += int((far & (dst == rank)).sum())
            captured.clear()
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            go(0)
            e.record()
            e.synchronize()
            ep.check()
            v = torch.tensor([s.elapsed_time(e) * 1000.0 / (len(batches) * args.layers),
                              sum(rows) / len(rows), local / max(remote, 1)], device=dev)
            vmax = v.clone()
            all_reduce(vmax, op=dist.ReduceOp.MAX)
            all_reduce(v)
            out = {"case": name, "mode": label, "tokens_per_rank": T, "n_gpus": world, "layers": args.layers,
                   "fp8": args.fp8, "zipf": args.zipf, "us_per_layer": round(float(vmax[0]), 1),
                   "remote_rows_per_token": round(float(v[1]) / world, 3),
                   "choices_served_locally_by_cache": round(float(v[2]) / world, 3)}
            return out

        with torch.no_grad():
            res = [measure("plain")]
            enable_speculation(model, args.slots, predictor=args.predictor, interval=args.interval)
            r = measure(f"speculative_slots{args.slots}_{args.predictor}_every{args.interval}")
            st = torch.zeros(4, dtype=torch.int64, device=dev)
            for layer in model.layers:
                st += layer.spec.cache.stats
            all_reduce(st)
            h, f = int(st[0]), int(st[1])
            r.update(cache_hits=h, cache_fetches=f, hit_rate=round(h / max(h + f, 1), 3))
            res.append(r)
        for layer in model.layers:
            if layer.spec is not None:
                layer.spec.close()
        ep.close()
        return res

    results = []
    if "prefill" in args.cases:
        results += run_case("prefill", 8192, 1)
    if "decode" in args.cases:
        results += run_case("decode", 128, args.decode_steps)
    if rank == 0:
        for r in results:
            print(json.dumps(r), flush=True)
    if multi:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
