"""Run warm-up training steps, then exactly one step between cudaProfilerStart/Stop.

Meant for ``ncu --profile-from-start off ...`` (launch list / kernel captures, one GPU) or
for a plain timing of one step; under torchrun it runs expert-parallel over all ranks and
rank 0 prints its per-kernel table.

    python benchmarks/profile_step.py --layers 8 [--warmup 2]
    python benchmarks/profile_step.py --layers 48 --table   # per-kernel device time (torch profiler)
    python benchmarks/profile_step.py --layers 48 --breakdown   # device time per kernel class
    python benchmarks/profile_step.py --layers 48 --gaps        # device idle gaps by size
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/profile_step.py --layers 48 --table --expert-state fp32

``--breakdown`` groups every kernel of one step by class (expert GEMMs, attention, dense
GEMMs, optimizer, EP data plane, elementwise, collectives, other) and reports the
device time of each class, the sum, and the step's wall time on the device minus that
sum (launch gaps and waits; kernels on side streams can overlap, so the gap may be
negative).
"""
import argparse
import os
import re
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

# (class, regex over the kernel name); first match wins
CLASSES = [
    ("ep: plan/dispatch/combine", r"route_plan|route_tables|dispatch_kernel|recv_|combine_kernel|source_reduce|"
                                  r"wait_rows|count_publish"),
    ("expert grouped GEMM (tcgen05)", r"gg_kernel|grouped_gemm|GroupedGemm|gemm_kernel<"),
    ("attention fwd", r"attn_fwd|attention_fwd|flash_fprop|sdpa.*fprop|fmha.*fwd|flash_fwd"),
    ("attention bwd", r"attn_bwd|attention_bwd|bprop|fmha.*bwd|flash_bwd|dot_do_o|convert_dq"),
    ("dense GEMM (tcgen05)", r"dense_gemm|linear_kernel"),
    ("dense GEMM (cuBLAS)", r"nvjet|cutlass|gemm|sm100_xmma|cublas"),
    ("optimizer", r"adamw|adam"),
    ("norm / rope / router / swiglu / xent", r"rmsnorm|rope|router|swiglu|xent|qk_norm"),
    ("collectives (NCCL)", r"nccl"),
    ("copies / fills / casts", r"elementwise_kernel|vectorized_elementwise|unrolled_elementwise|fill|copy|Memcpy|"
                               r"Memset|reduce_kernel|index|scatter|gather|cat|embedding"),
]


def classify(name: str) -> str:
    for cls, pat in CLASSES:
        if re.search(pat, name, re.I):
            return cls
    return "other"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--expert-state", default="8bit")
    ap.add_argument("--table", action="store_true", help="print per-kernel CUDA time of one step (torch profiler)")
    ap.add_argument("--breakdown", action="store_true", help="print device time per kernel class of one step")
    ap.add_argument("--gaps", action="store_true",
                    help="list the device idle gaps of one step (between consecutive kernels) by size")
    ap.add_argument("--out", default=None, help="also write the breakdown (markdown) to this file")
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
    # different tokens on every rank (as in bench.py): identical batches would route every
    # rank's copy of a token to the same experts and pile the rows onto a few ranks
    gen = torch.Generator().manual_seed(rank)
    ids = torch.randint(0, cfg.vocab_size, (1, args.seq), generator=gen).to(dev)
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
    step_ms = s.elapsed_time(e)
    if rank == 0:
        print(f"world={world} layers={args.layers} step_ms={step_ms:.2f} loss={loss.item():.4f}")
    if args.table or args.breakdown or args.gaps:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            tr.train_step(ids, lab, args.seq - 1)
            torch.cuda.synchronize()
        if rank == 0 and args.table:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=90))
        if rank == 0 and args.breakdown:
            text = breakdown(prof, step_ms, world, args)
            print(text)
            if args.out:
                with open(args.out, "w") as f:
                    f.write(text + "\n")
        if rank == 0 and args.gaps:
            text = gaps(prof)
            print(text)
            if args.out:
                with open(args.out, "a") as f:
                    f.write("\n" + text + "\n")
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def gaps(prof, top=20) -> str:
    """Device idle time of the profiled step: kernels (and memcpy / memset) sorted by start,
    idle = time between the latest end so far and the next start. Lists the size histogram
    and the largest gaps with the kernels on either side."""
    evs = []
    for ev in prof.events():
        if getattr(ev, "device_type", None) is None or str(ev.device_type) != "DeviceType.CUDA":
            continue
        tr = ev.time_range
        if tr.end > tr.start:
            evs.append((tr.start, tr.end, ev.name))
    evs.sort()
    if not evs:
        return "no device events"
    found, end, prev = [], evs[0][1], evs[0][2]
    for st, en, name in evs[1:]:
        if st > end:
            found.append((st - end, prev, name))
        if en > end:
            end, prev = en, name
    span = end - evs[0][0]
    idle = sum(g for g, _, _ in found)
    bins = [(0, 5), (5, 20), (20, 100), (100, 1000), (1000, float("inf"))]
    lines = [f"device span {span / 1e3:.2f} ms, idle {idle / 1e3:.2f} ms in {len(found)} gaps", "",
             "| gap size (us) | gaps | idle ms |", "|---|---|---|"]
    for lo, hi in bins:
        sel = [g for g, _, _ in found if lo <= g < hi]
        lines.append(f"| {lo}-{hi if hi != float('inf') else ''} | {len(sel)} | {sum(sel) / 1e3:.2f} |")
    lines += ["", "| gap (us) | after | before |", "|---|---|---|"]
    for g, a, b in sorted(found, reverse=True)[:top]:
        lines.append(f"| {g:.1f} | {a[:60]} | {b[:60]} |")
    return "\n".join(lines)


def breakdown(prof, step_ms, world, args) -> str:
    per_cls: dict[str, list] = {}
    for ev in prof.key_averages():
        us = ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
        if us <= 0:
            continue
        c = classify(ev.key)
        d = per_cls.setdefault(c, [0.0, 0, []])
        d[0] += us
        d[1] += ev.count
        d[2].append((us, ev.count, ev.key))
    total_us = sum(v[0] for v in per_cls.values())
    lines = [f"one training step, {args.model}, {args.layers} layers, seq {args.seq}, world {world}, "
             f"expert state {args.expert_state}",
             f"step (CUDA events, unprofiled run): {step_ms:.2f} ms; kernel time summed: {total_us / 1e3:.2f} ms; "
             f"step minus kernel sum: {step_ms - total_us / 1e3:.2f} ms",
             "", "| class | ms / step | share of kernel time | launches | top kernels (ms) |", "|---|---|---|---|---|"]
    for c, (us, n, ks) in sorted(per_cls.items(), key=lambda kv: -kv[1][0]):
        ks.sort(reverse=True)
        top = "; ".join(f"{k[:60]} {u / 1e3:.2f}" for u, _, k in ks[:3])
        lines.append(f"| {c} | {us / 1e3:.2f} | {100 * us / max(total_us, 1):.1f}% | {n} | {top} |")
    # the kernels of the largest class by full template name (instances differ by tile
    # width, stage count, operand majorness and epilogue)
    big = max(per_cls.items(), key=lambda kv: kv[1][0])
    lines += ["", f"{big[0]}, per kernel:", "", "| kernel | ms / step | launches |", "|---|---|---|"]
    for u, cnt, k in sorted(big[1][2], reverse=True)[:10]:
        name = k.split("(")[0].replace("void ", "").replace("sepx::", "")
        lines.append(f"| `{name}` | {u / 1e3:.2f} | {cnt} |")
    return "\n".join(lines)


if __name__ == "__main__":
    main()
