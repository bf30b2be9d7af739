"""MoE model driver (reference: scripts/ds_moe.py).

Builds a Qwen3-MoE-shaped model behind the DeepSpeed-style ``initialize`` of
``spec_ep.integrations.ds_moe`` (random init: no checkpoint or dataset is needed), gives
every rank a disjoint ``seq_len`` slice of token ids, and runs the requested modes:

  latency   forward latency, CUDA events between barrier+synchronize, max over ranks
  routing   records every layer's top-k expert ids -> $LOGS/experts_rank{r}.pt ([L, T, K] int16)
  profile   torch.profiler trace per rank -> $LOGS/profile/trace_rank{r}.json
  flops     analytic FLOPs and achieved TFLOP/s of one forward
  comm      per-op device time / bytes of the EP dispatch+combine (max over ranks)
  train     timed training steps (forward + backward + AdamW)

``--speculative-slots N`` turns on speculative expert replication (an LRU cache of N
predicted-hot experts per layer and rank; inference modes only) and prints the cache
statistics at the end.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/ds_moe.py \
        --config-pth configs/qwen3_30b_a3b_ep8_sepx.json --modes latency flops routing
"""
import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from spec_ep.integrations.ds_moe import initialize  # noqa: E402
from spec_ep.utils.dist import init_distributed, print0, shutdown_comm  # noqa: E402
from spec_ep.utils.metrics import max_over_ranks  # noqa: E402
from spec_ep.utils.profile import (FlopCounter, RoutingRecorder, add_expert_statistics_hook, count_params,  # noqa: E402
                                   end_flops_profile, record_function, report_peak_mem, save_torch_profile,
                                   start_flops_profile, torch_profile_ctx)


def get_batch(vocab, rank, seq_len, device, text_ids=None):
    if text_ids is not None:  # disjoint slice of a pre-tokenised corpus, like the reference
        s, e = rank * seq_len, (rank + 1) * seq_len
        if text_ids.numel() < e:
            raise ValueError(f"Provide more text: at least {e} tokens are required.")
        ids = text_ids[s:e]
    else:
        g = torch.Generator().manual_seed(rank)
        ids = torch.randint(0, vocab, (seq_len,), generator=g)
    ids = ids.view(1, -1).to(device)
    labels = torch.cat([ids[:, 1:], torch.full((1, 1), -1, device=device)], 1).int()
    return ids, labels


def timed(fn, dev):
    torch.cuda.synchronize(dev)
    if dist.is_initialized():
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    out = fn()
    e.record()
    torch.cuda.synchronize(dev)
    return max_over_ranks({"ms": s.elapsed_time(e)}, dev)["ms"], out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config-pth", default="configs/qwen3_30b_a3b_ep8_sepx.json")
    ap.add_argument("--model", default="qwen3-30b-a3b", help="spec_ep preset")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--modes", nargs="+", default=["latency", "flops"])
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--speculative-slots", type=int, default=0)
    args, _ = ap.parse_known_args()  # launchers may inject --local_rank
    rank, world, dev = init_distributed()
    logs = Path(os.environ.get("LOGS", f"logs/{time.strftime('%Y-%m-%d_%H-%M-%S')}"))
    logs.mkdir(parents=True, exist_ok=True)
    cfg = json.load(open(args.config_pth))
    cfg["expert_parallel"]["autoep_size"] = min(cfg["expert_parallel"].get("autoep_size", world), world)
    if args.speculative_slots:
        cfg["expert_parallel"].setdefault("sepx", {})["speculative_slots"] = args.speculative_slots
        if "train" in args.modes:
            raise SystemExit("speculative replication is inference-only: drop the train mode")
    from spec_ep.models import config as mc

    if args.layers:
        mc.PRESETS[args.model] = mc.get_config(args.model, num_layers=args.layers)
    engine, opt, _, _ = initialize(model=args.model, config=cfg, max_tokens=args.seq_len, device=dev)
    total, expert = count_params(engine.module)
    print0(f"local params: {total / 1e9:.2f}B ({expert / 1e9:.2f}B in experts)")
    ids, labels = get_batch(engine.module.cfg.vocab_size, rank, args.seq_len, dev)

    if "latency" in args.modes:
        with torch.no_grad():
            engine(ids)
            ms, _ = timed(lambda: engine(ids), dev)
        print0(f"forward latency (max over ranks): {ms:.2f} ms")
    if "routing" in args.modes:
        rec = RoutingRecorder()
        add_expert_statistics_hook(engine.module, rec)
        with torch.no_grad():
            engine(ids)
        print0(f"routing saved: {rec.save(logs)}")
        for layer in engine.module.layers:
            layer.routing_callback = None
    if "profile" in args.modes:
        with torch_profile_ctx() as prof:
            with record_function("forward"), torch.no_grad():
                engine(ids)
            torch.cuda.synchronize(dev)
        print0(f"trace: {save_torch_profile(prof, logs, verbose=True)}")
    if "flops" in args.modes:
        fc = FlopCounter(engine.module.cfg, args.seq_len, args.seq_len)
        with torch.no_grad():
            ms, _ = timed(lambda: engine(ids), dev)
            prof = start_flops_profile(engine, args.seq_len, args.seq_len)
            engine(ids)
            path = end_flops_profile(prof, logs)
        print0(f"forward: {fc.step_flops(False) / 1e12:.1f} TFLOP/rank, {fc.tflops(ms, False):.0f} TFLOP/s per GPU "
               f"(breakdown: {path})")
    if "comm" in args.modes:
        ep = engine.ep
        x = torch.randn(args.seq_len, engine.module.cfg.hidden_size, device=dev).bfloat16()
        te = torch.randint(0, ep.E, (args.seq_len, ep.k), device=dev).int()
        tw = torch.full((args.seq_len, ep.k), 1.0 / ep.k, device=dev)
        ms_d, st = timed(lambda: ep.dispatch_fwd(x, te, tw), dev)
        ms_c, _ = timed(lambda: ep.combine_fwd(st.xp, st), dev)
        print0(f"dispatch {ms_d * 1e3:.0f} us, combine {ms_c * 1e3:.0f} us (max over ranks)")
    if "train" in args.modes:
        for _ in range(2):
            engine.train_step(ids, labels, args.seq_len - 1)
        ms, loss = timed(lambda: [engine.train_step(ids, labels, args.seq_len - 1) for _ in range(args.steps)][-1], dev)
        print0(f"train step {ms / args.steps:.1f} ms, {world * args.seq_len / (ms / args.steps / 1e3):.0f} tokens/s, "
               f"loss {float(loss):.3f}")
    if args.speculative_slots:
        from spec_ep.parallel.speculative import speculation_summary

        print0(f"speculative replication: {speculation_summary(engine.module)}")
    report_peak_mem(dev)
    engine.ep.close()
    shutdown_comm()


if __name__ == "__main__":
    main()
