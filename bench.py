#!/usr/bin/env python
"""Flagship benchmark: Qwen3-30B-A3B-shaped MoE training step with expert parallelism.

    python bench.py [--gpus N --steps K --warmup W]                 # this framework
    python bench.py --impl reference [--gpus N ...]                 # the reference arm
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step = forward + backward + dense-gradient all-reduce + AdamW on 4096 tokens per GPU
(micro-batch 1, seq 4096), 48 layers, 128 experts top-8, EP = number of GPUs. The timed
region covers exactly K steps between barrier + synchronize brackets, timed with CUDA
events and reduced with MAX over ranks. ``value`` is total tokens/s of the job.

The end-to-end number (``e2e``) runs the same steps through ``Trainer.train_step_from_host``:
every step copies its token ids and labels from pinned host memory and reads the loss
back to the host.

``dispatch_combine_us_per_layer`` is measured separately on the MoE-layer shape
(hidden 2048, 4096 tokens/rank, 128 experts, top-8, Zipf s=1.0 routing) with identity
experts, so it is the pure dispatch+combine cost, on the contiguous expert layout the
reference uses; it is the mean over routing seeds 0-4 (per-seed values alongside), each
layer call launched from the host as the training step does. ``..._graph`` replays the
seed-0 layer from a CUDA graph: the device time alone, without per-call host cost.

``check`` is a correctness figure taken on the same ranks before anything is timed: one
small expert-parallel MoE forward + backward (512 tokens/rank, 16 experts, top-4, hidden
512) through the fused kernels against an fp32 PyTorch MoE holding all experts; the
largest relative error of the output and of every gradient, max over ranks.

The expert optimizer state is block-wise 8-bit at every world size by default (the only
precision that fits all experts of the model on one GPU), so every point of the scaling
curve runs the same optimizer; ``--expert-state fp32`` selects fp32 state where it fits. ``dispatch_combine_us_per_layer_planned`` repeats it with the
speculative placement: experts packed by the load of a *previous* batch's routing (seed
1) and the 16 hottest replicated on every rank, measured on the seed-0 batch.

``roofline`` gives both measured times as fractions of their bounds (the slowest of
compute at the measured bf16 peak, minimum HBM bytes at the measured copy bandwidth and
NVLink bytes at the measured peer bandwidth; ``spec_ep.utils.roofline``).
"""
from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE dispatch+combine µs/layer & train tokens/sec, Qwen3-30B-A3B EP=1/2/4/8"


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["spec_ep", "reference"], default="spec_ep")
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--layers", type=int, default=None, help="override depth (smoke runs only; invalid for the bench)")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--micro-batch", type=int, default=1)
    ap.add_argument("--expert-state", choices=["auto", "fp32", "8bit"], default="8bit",
                    help="expert optimizer state; 8bit (default) at every N keeps the scaling curve like for like")
    ap.add_argument("--dc-iters", type=int, default=20)
    ap.add_argument("--ep", type=int, default=None,
                    help="expert-parallel group size (default: every GPU); world / ep expert-data-parallel "
                         "replicas, e.g. --gpus 8 --ep 4 for EP=4 x DP=2")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    return world, rank, dev


def max_over_ranks(x: float, dev) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_clocks(summary: dict):
    if not dist.is_initialized():
        return summary
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, summary)
    mhz = [s["sm_mhz"] for s in out if s.get("sm_mhz") is not None]
    reasons = sorted({r for s in out for r in s.get("reasons", [])})
    return {"sm_mhz": min(mhz) if mhz else None,
            "sm_max_mhz": max((s["sm_max_mhz"] or 0) for s in out) or None,
            "reasons": reasons, "per_rank_sm_mhz": [s.get("sm_mhz") for s in out]}


def timed(fn, steps, dev):
    """Run fn() `steps` times between barrier+sync brackets; CUDA-event ms/step, max over ranks."""
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    if dist.is_initialized():
        dist.barrier()
    return max_over_ranks(s.elapsed_time(e) / steps, dev)


def gpu_uuid(dev):
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ---------------------------------------------------------------------------------------
def dispatch_combine_us(ep, dev, rank, world, iters, seeds=(0, 1, 2, 3, 4)):
    """Identity-expert dispatch + combine on the MoE-layer shape, max over ranks, for each
    routing seed; returns (mean µs, per-seed µs, rows per token of seed 0)."""
    from spec_ep.utils.routing import dedup_bound_rows, synthetic_routing

    per_seed, bound = [], None
    for seed in seeds:
        x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=seed, rank=rank, device=dev)

        def once():  # one layer call per pass, with the row budget the training step uses
            ep.begin_pass()
            st = ep.dispatch_fwd(x, te, tw)
            ep.combine_fwd(st.xp, st)

        for _ in range(3):
            once()
        ep.end_pass()  # learn / verify the budget before timing
        per_seed.append(timed(once, iters, dev) * 1000.0)
        if ep.end_pass():
            raise RuntimeError("a dispatch outgrew its row budget inside the timed loop")
        ep.check()
        if bound is None:
            bound = dedup_bound_rows(te.cpu(), 128 // world, rank, world)
    return sum(per_seed) / len(per_seed), per_seed, bound


def dispatch_combine_graph_us(ep, dev, rank, iters):
    """The same layer (seed 0) captured once in a CUDA graph and replayed: the device time
    of dispatch + combine without the host's per-call launch cost (what the layer costs
    inside a step whose host runs ahead of the GPU). Row budget as in training."""
    from spec_ep.parallel.ep import EPGraph
    from spec_ep.utils.routing import synthetic_routing

    x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=0, rank=rank, device=dev)

    def once():
        ep.begin_pass()
        st = ep.dispatch_fwd(x, te, tw)
        out = ep.combine_fwd(st.xp, st)
        ep._pass = None  # the replays run no host code; the miss flag is read below
        return out

    once()
    ep.end_pass()
    g = EPGraph(ep, once)
    us = timed(g.replay, iters, dev) * 1000.0
    torch.cuda.synchronize(dev)
    missed = int(ep._miss.item())
    del g
    ep.graph_epochs(False)
    ep.check()
    if missed:
        raise RuntimeError("a graph-replayed dispatch outgrew its row budget")
    return us


def dispatch_combine_planned_us(dev, rank, world, iters):
    """Same layer with the placement planned from the previous batch's expert loads."""
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.parallel.placement import plan_balanced
    from spec_ep.utils.routing import synthetic_routing

    _, te_prev, _ = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=1, rank=rank, device=dev)
    load = torch.bincount(te_prev.flatten().long(), minlength=128).float()
    if dist.is_initialized():
        dist.all_reduce(load)
    placement = plan_balanced(load.cpu(), world, replicate_top=16 if world > 1 else 0)
    ep = ExpertParallel(128, 8, 2048, max_tokens=4096, device=dev, placement=placement)
    x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=0, rank=rank, device=dev)

    def once():
        ep.begin_pass()
        st = ep.dispatch_fwd(x, te, tw)
        ep.combine_fwd(st.xp, st)

    for _ in range(3):
        once()
    ep.end_pass()
    ms = timed(once, iters, dev)
    if ep.end_pass():
        raise RuntimeError("a dispatch outgrew its row budget inside the timed loop")
    ep.check()
    ep.close()
    return ms * 1000.0


def run_spec_ep(args):
    world, rank, dev = init_dist()
    from spec_ep.models.config import get_config
    from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
    from spec_ep.ops._ext import load
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.train import Trainer, choose_state_precision
    from spec_ep.utils.clocks import ClockSampler

    C = load()
    from spec_ep.utils.selfcheck import ep_moe_check

    check = ep_moe_check(dev)  # correctness on these ranks, before anything is timed
    cfg = get_config(args.model)
    if args.layers:
        cfg.num_layers = args.layers
    T = args.seq * args.micro_batch
    ep_size = args.ep or world
    ep_group = dp_group = None
    if ep_size != world:
        from spec_ep.integrations.ds_moe import make_groups

        ep_group, dp_group = make_groups(ep_size)
    ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=T, device=dev, group=ep_group)
    total, expert = cfg.param_counts()
    dense = total - expert
    local_expert = expert // ep_size
    # saved activations per layer: ~12 [T, H] tensors + the expert rows (x and gate|up),
    # with 1.5x headroom for routing imbalance
    rows = int(1.5 * T * cfg.top_k) + ep.G * 64
    act = cfg.num_layers * (T * cfg.hidden_size * 2 * 12 + rows * (cfg.hidden_size + 2 * cfg.moe_intermediate_size) * 2)
    budget = int(0.92 * torch.cuda.get_device_properties(dev).total_memory)
    prec = args.expert_state
    if prec == "auto":
        prec = choose_state_precision(local_expert, dense, budget, act + (4 << 30))
    torch.manual_seed(1234)  # same dense init on every rank (replicated weights)
    model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
    trainer = Trainer(model, lr=1e-4, expert_state=prec, expert_dp_group=dp_group)

    g = torch.Generator().manual_seed(rank)
    ids_cpu = torch.randint(0, cfg.vocab_size, (args.micro_batch, args.seq), generator=g)
    lab_cpu = torch.cat([ids_cpu[:, 1:], torch.full((args.micro_batch, 1), -1)], 1).int()
    ids_cpu, lab_cpu = ids_cpu.pin_memory(), lab_cpu.pin_memory()
    num_valid = args.micro_batch * (args.seq - 1)
    ids, lab = ids_cpu.to(dev), lab_cpu.to(dev)

    for _ in range(args.warmup):
        trainer.train_step(ids, lab, num_valid)
    torch.cuda.synchronize(dev)
    ep.check()

    launches0 = C.launch_count()
    retries0 = trainer.budget_retries
    with ClockSampler(gpu_uuid(dev)) as clk:
        ms = timed(lambda: trainer.train_step(ids, lab, num_valid), args.steps, dev)
    launches = (C.launch_count() - launches0)
    retries_timed = trainer.budget_retries - retries0
    clocks = gather_clocks(clk.summary())
    ep.check()
    loss_dev = float(trainer.train_step(ids, lab, num_valid).item())
    tokens = world * T
    value = tokens / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        losses = []
        with ClockSampler(gpu_uuid(dev)) as clk_e2e:
            e2e_ms = timed(lambda: losses.append(trainer.train_step_from_host(ids_cpu, lab_cpu, num_valid)),
                           args.steps, dev)
        e2e_clocks = gather_clocks(clk_e2e.summary())
        e2e = {"value": tokens / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "clocks": e2e_clocks,
               "h2d_bytes_per_step": ids_cpu.numel() * ids_cpu.element_size() + lab_cpu.numel() * lab_cpu.element_size(),
               "d2h_bytes_per_step": 4, "api": "spec_ep.train.Trainer.train_step_from_host",
               "last_loss": losses[-1] if losses else None}

    dc_us, dc_seeds, bound = dispatch_combine_us(ep, dev, ep.rank, ep.world, args.dc_iters)
    dc_graph_us = dispatch_combine_graph_us(ep, dev, ep.rank, args.dc_iters)
    dc_planned_us = dispatch_combine_planned_us(dev, rank, world, args.dc_iters) if ep_size == world else None
    peak = torch.cuda.max_memory_allocated(dev) / 2**30
    peak = max_over_ranks(peak, dev)
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids, random-init weights)",
            "config": {"model": "Qwen3-30B-A3B", "global_batch": world * args.micro_batch, "seq_len": args.seq,
                       "parallelism": (f"ep{ep_size}" + (f"xdp{world // ep_size}(experts)" if ep_size != world else "")
                                       + (f"+dp{world}(dense)" if world > 1 else "")),
                       "layers": cfg.num_layers, "experts": cfg.num_experts, "top_k": cfg.top_k,
                       "hidden": cfg.hidden_size, "moe_inter": cfg.moe_intermediate_size,
                       "optimizer": "AdamW (dense: fp32 master+moments; experts: %s state at every N, updated "
                                    "in backward)" % prec,
                       "l2": "no flush: every step streams > 60 GB of weights and optimizer state (>> 126 MB L2)",
                       "attention": "torch SDPA (GQA, causal)"},
            "impl": "spec_ep",
            "dispatch_combine_us_per_layer": dc_us,
            "dispatch_combine_us_per_seed": dc_seeds,
            "dispatch_combine_us_per_layer_graph": dc_graph_us,
            "dispatch_combine_shape": "hidden 2048, 4096 tok/rank, 128 experts, top-8, Zipf s=1.0 (seeds 0-4), "
                                      "identity experts",
            "dispatch_combine_us_per_layer_planned": dc_planned_us,
            "check": {"what": "ep_moe fwd+bwd, 512 tok/rank, 16 experts, top-4, hidden 512, vs fp32 torch MoE; "
                              "max relative error over ranks",
                      **check},
            "check_max_rel_err": check["max"],
            "planned_placement": "LPT packing of the previous batch's loads + top-16 experts replicated on every rank",
            "rows_per_token": bound,
            "loss": loss_dev, "peak_mem_gib": peak,
            "row_budget_retries": {"total": trainer.budget_retries, "in_timed_steps": retries_timed,
                                   "what": "forwards run again because an MoE layer's received rows outgrew the "
                                           "row budget its buffers were sized with (counted, and timed, as "
                                           "part of the step)"},
            "gpu_launches": launches, "clocks": clocks, "e2e": e2e,
        }
        try:  # fraction of roofline (CPU arithmetic after the timed regions)
            from spec_ep.utils.roofline import bench_fields

            out["roofline"] = bench_fields(cfg, T, args.seq, world, prec, ms, dc_us,
                                           os.path.join(ROOT, "MEASURED_PEAKS.json"))
        except Exception as e:  # the analysis must never cost the measured line
            out["roofline"] = {"error": f"{type(e).__name__}: {e}"}
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
def _load_reference_rbd():
    path = os.path.join(ROOT, "baseline", "_ref", "spec_ep", "rbd.py")
    if not os.path.exists(path):
        return None, f"reference not installed at {path}"
    spec = importlib.util.spec_from_file_location("reference_spec_ep_rbd", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, None


def run_reference(args):
    """The reference's own stock path: spec_ep.rbd.RBD_combine_dispatch over NCCL.

    The reference has no training step (its RBD is forward-only, src/rbd.py:25-26, and its
    model driver is inference-only under DeepSpeed AutoEP, which is not installed), so the
    training metric is reported unavailable; the dispatch+combine cost per layer is
    measured on the same shape and routing as this framework's arm.
    """
    world, rank, dev = init_dist()
    rbd, err = _load_reference_rbd()
    reason = ("train tokens/s: the reference has no training path (RBD has no backward, src/rbd.py:25-26; "
              "its model driver scripts/ds_moe.py is inference-only and needs DeepSpeed AutoEP, not installed)")
    if rbd is None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": err}), flush=True)
        return
    from spec_ep.utils.routing import synthetic_routing

    if world == 1:
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:29593", rank=0, world_size=1, device_id=dev)
    local_group, _ = dist.new_subgroups(group_size=world)
    per_seed = []
    for seed in range(5):
        x, te, tw = synthetic_routing(4096, 2048, 128, 8, s=1.0, seed=seed, rank=rank, device=dev)

        def once():
            rbd.RBD_combine_dispatch(x, tw, lambda rows, ids: rows, te.long(), E=128, gpus_per_node=world,
                                     local_group=local_group, concurrent=True)

        for _ in range(3):
            once()
        per_seed.append(timed(once, args.dc_iters, dev) * 1000.0)
    if rank == 0:
        rec = reference_record(world, sum(per_seed) / len(per_seed), reason)
        rec["dispatch_combine_us_per_seed"] = per_seed
        print(json.dumps(rec), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def reference_record(world: int, dispatch_combine_us: float, reason: str) -> dict:
    """The reference arm's JSON line: its dispatch+combine time on this framework's layer
    shape; the training metric is unavailable for the given reason."""
    return {
        "impl": "reference", "metric": METRIC, "unavailable": reason, "n_gpus": world,
        "dispatch_combine_us_per_layer": dispatch_combine_us,
        "dispatch_combine_shape": "hidden 2048, 4096 tok/rank, 128 experts, top-8, Zipf s=1.0 (seeds 0-4), "
                                  "identity experts",
        "api": "spec_ep.rbd.RBD_combine_dispatch (reference, unmodified, NCCL)",
    }


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_spec_ep(a)
