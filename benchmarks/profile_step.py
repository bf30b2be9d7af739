"""Run warm-up training steps, then exactly one step between cudaProfilerStart/Stop.

Meant for ``ncu --profile-from-start off ...`` (launch list / kernel captures, one GPU) or
for a plain timing of one step; under torchrun it runs expert-parallel over all ranks and
rank 0 prints its per-kernel table.

    python benchmarks/profile_step.py --layers 8 [--warmup 2]
    python benchmarks/profile_step.py --layers 48 --table   # per-kernel device time (torch profiler)
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/profile_step.py --layers 48 --table --expert-state fp32
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--expert-state", default="8bit")
    ap.add_argument("--table", action="store_true", help="print per-kernel CUDA time of one step (torch profiler)")
    args = ap.parse_args()
    from spec_ep.models.config import get_config
    from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.train import Trainer

    from spec_ep.utils.dist import init_distributed

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        rank, world, dev = init_distributed()
    else:
        rank, world, dev = 0, 1, torch.device("cuda", 0)
        torch.cuda.set_device(dev)
    cfg = get_config(args.model, num_layers=args.layers)
    ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=args.seq, device=dev)
    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
    tr = Trainer(model, lr=1e-4, expert_state=args.expert_state)
    ids = torch.randint(0, cfg.vocab_size, (1, args.seq), device=dev)
    lab = torch.cat([ids[:, 1:], torch.full((1, 1), -1, device=dev)], 1).int()
    for _ in range(args.warmup):
        tr.train_step(ids, lab, args.seq - 1)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    s.record()
    loss = tr.train_step(ids, lab, args.seq - 1)
    e.record()
    torch.cuda.profiler.stop()
    torch.cuda.synchronize()
    ep.check()
    if rank == 0:
        print(f"world={world} layers={args.layers} step_ms={s.elapsed_time(e):.2f} loss={loss.item():.4f}")
    if args.table:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            tr.train_step(ids, lab, args.seq - 1)
            torch.cuda.synchronize()
        if rank == 0:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=70))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
