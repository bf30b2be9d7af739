"""Training launcher: the step loop around ``Trainer`` with metrics, checkpoints and resume.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m spec_ep.run \\
        --model qwen3-30b-a3b --steps 200 --log-dir logs/run1 --ckpt-every 100 [--resume logs/run1/step_100]

Every step copies its batch from pinned host memory, runs ``Trainer.train_step`` and
reads the loss back. Each rank appends a JSON line per step to
``<log-dir>/metrics_rank{r}.jsonl`` (loss, device ms, job tokens/s, and with
``--ep-stats`` the expert-parallel traffic: rows sent per token through the per-rank
dedup, the per-copy count a plain all-to-all would send, and the received-row imbalance
max / mean over ranks). Rank 0 prints the same line with timings maxed over ranks.

Data: ``--token-file`` is a flat binary array of token ids (``--token-dtype`` uint16 /
uint32 / int32); step s of rank r reads the disjoint window number ``s * world + r``, as
the reference gives each rank its own slice of one text (scripts/ds_moe.py:64-87).
Without a file the batches are uniform random ids drawn from a generator seeded by
(seed, rank, step), so a resumed run sees the same batches as an uninterrupted one.

The loop itself (``train_loop``) takes any object with ``train_step_from_host`` and
runs on CPU too; ``main`` builds the Qwen3-MoE model on the GPUs.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch
import torch.distributed as dist


class TokenBatches:
    """Deterministic per-(rank, step) batches of ``[micro_batch, seq]`` token ids + labels."""

    def __init__(self, vocab, seq, micro_batch, rank, world, seed=0, token_file=None, token_dtype="uint32",
                 pin=True):
        self.vocab, self.seq, self.mb, self.rank, self.world, self.seed = vocab, seq, micro_batch, rank, world, seed
        self.pin = pin and torch.cuda.is_available()
        self.tokens = None
        if token_file is not None:
            self.tokens = np.memmap(token_file, dtype=np.dtype(token_dtype), mode="r")
            need = micro_batch * seq + 1
            if self.tokens.shape[0] < need:
                raise ValueError(f"{token_file} holds {self.tokens.shape[0]} tokens, one batch needs {need}")

    def get(self, step: int):
        n = self.mb * self.seq
        if self.tokens is not None:
            windows = (self.tokens.shape[0] - 1) // n
            w = (step * self.world + self.rank) % windows
            flat = torch.from_numpy(np.asarray(self.tokens[w * n:(w + 1) * n + 1], dtype=np.int64))
            if int(flat.max()) >= self.vocab:
                raise ValueError(f"token id {int(flat.max())} is outside the vocabulary ({self.vocab})")
            ids = flat[:-1].view(self.mb, self.seq)
            labels = flat[1:].view(self.mb, self.seq).int()
        else:
            g = torch.Generator().manual_seed((self.seed * 1_000_003 + self.rank) * 1_000_003 + step)
            ids = torch.randint(0, self.vocab, (self.mb, self.seq), generator=g)
            labels = torch.cat([ids[:, 1:], torch.full((self.mb, 1), -1)], 1).int()
        if self.pin:
            ids, labels = ids.pin_memory(), labels.pin_memory()
        return ids, labels


def _timer():
    if torch.cuda.is_available():
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()

        def stop():
            e.record()
            e.synchronize()
            return s.elapsed_time(e)
    else:
        t0 = time.perf_counter()

        def stop():
            return (time.perf_counter() - t0) * 1000.0
    return stop


def _reduce(values: list[float], op, device):
    if not (dist.is_available() and dist.is_initialized()):
        return values
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return t.tolist()


def train_loop(trainer, batches: TokenBatches, steps: int, start_step: int = 0, log_dir=None, ckpt_every: int = 0,
               save_fn=None, ep=None, print_fn=print, num_valid=None, heartbeat=None, timeline=None):
    """Run steps ``start_step .. steps-1``; returns the per-step records of this rank.

    ``save_fn(path, step)`` is called (on every rank: it is collective) after every
    ``ckpt_every`` steps with ``<log_dir>/step_<n>``. With a ``heartbeat``
    (``spec_ep.utils.heartbeat.Heartbeat``), every step starts with a host-side arrival
    that waits for all peers to arrive too (``PeerLostError`` names a lost rank before
    this rank launches anything); steps count from ``start_step``. With a ``timeline``
    (``spec_ep.utils.trace.DeviceTimeline``), every EP stage of the step (dispatch,
    experts, combine and their backward halves) is stamped on the device and the record
    gets ``stage_us``: per stage, the mean device µs per layer call and the call count.
    """
    from .utils.trace import enable_stage_timeline

    rank = dist.get_rank() if (dist.is_available() and dist.is_initialized()) else 0
    world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
    device = ep.device if ep is not None else (torch.device("cuda", torch.cuda.current_device())
                                              if torch.cuda.is_available() else torch.device("cpu"))
    f = None
    if log_dir is not None:
        os.makedirs(log_dir, exist_ok=True)
        f = open(os.path.join(log_dir, f"metrics_rank{rank}.jsonl"), "a")
    if ep is not None:
        ep.enable_stats(True)
    records = []
    tokens_per_step = batches.mb * batches.seq
    try:
        for step in range(start_step, steps):
            if heartbeat is not None:
                heartbeat.arrive(step - start_step)
            ids, labels = batches.get(step)
            if timeline is not None:
                timeline.reset()
                enable_stage_timeline(timeline)
            stop = _timer()
            try:
                loss = trainer.train_step_from_host(ids, labels, num_valid)
            finally:
                if timeline is not None:
                    enable_stage_timeline(None)
            ms = stop()
            rec = {"ts": time.time(), "rank": rank, "step": step, "loss": loss, "ms": ms,
                   "tokens_per_s_rank": tokens_per_step / (ms / 1000.0)}
            if timeline is not None:
                rec["stage_us"] = {k: {"mean_us": v["mean_us"], "count": v["count"]}
                                   for k, v in timeline.durations().items()}
            if ep is not None:
                rec.update(ep.take_stats())
            if f is not None:
                f.write(json.dumps(rec) + "\n")
                f.flush()
            records.append(rec)
            # job view on rank 0: slowest rank's time, mean loss, received-row imbalance
            recv = rec.get("recv_rows_per_call", 0.0)
            mx = _reduce([ms, recv], dist.ReduceOp.MAX, device)
            sm = _reduce([loss, recv], dist.ReduceOp.SUM, device)
            if rank == 0 and print_fn is not None:
                job = {"step": step, "loss": sm[0] / world, "ms": mx[0],
                       "tokens_per_s": world * tokens_per_step / (mx[0] / 1000.0)}
                if ep is not None:
                    job.update(remote_rows_per_token=rec["remote_rows_per_token"],
                               naive_rows_per_token=rec["naive_rows_per_token"],
                               recv_imbalance=(mx[1] / (sm[1] / world)) if sm[1] > 0 else 1.0)
                print_fn(json.dumps(job))
            if ckpt_every and save_fn is not None and (step + 1) % ckpt_every == 0:
                save_fn(os.path.join(log_dir or ".", f"step_{step + 1}"), step + 1)
    finally:
        if f is not None:
            f.close()
        if ep is not None:
            ep.enable_stats(False)
    return records


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--micro-batch", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--lr", type=float, default=1e-4)
    ap.add_argument("--expert-state", choices=["auto", "fp32", "8bit"], default="auto")
    ap.add_argument("--token-file", default=None)
    ap.add_argument("--token-dtype", default="uint32")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--log-dir", default=None)
    ap.add_argument("--ckpt-every", type=int, default=0)
    ap.add_argument("--resume", default=None, help="checkpoint directory written by this launcher")
    ap.add_argument("--ep-stats", action="store_true")
    ap.add_argument("--stage-times", action="store_true",
                    help="stamp every EP stage on the device; per-stage µs per layer call in the metrics")
    ap.add_argument("--heartbeat-timeout", type=float, default=0.0,
                    help="seconds without progress after which a peer counts as lost (host check before "
                         "every step; set it above the longest step); 0 = off")
    args = ap.parse_args(argv)

    from . import checkpoint
    from .models.config import get_config
    from .models.qwen3_moe import Qwen3MoeForCausalLM
    from .parallel.ep import ExpertParallel
    from .train import Trainer, choose_state_precision
    from .utils.dist import init_distributed, shutdown_comm

    rank, world, dev = init_distributed(timeout_s=600)
    cfg = get_config(args.model)
    if args.layers:
        cfg.num_layers = args.layers
    T = args.seq * args.micro_batch
    ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=T, device=dev)
    prec = args.expert_state
    if prec == "auto":
        total, expert = cfg.param_counts()
        act = cfg.num_layers * T * cfg.hidden_size * 2 * 24
        prec = choose_state_precision(expert // world, total - expert,
                                      int(0.9 * torch.cuda.get_device_properties(dev).total_memory), act)
    torch.manual_seed(args.seed)  # replicated dense init
    model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
    trainer = Trainer(model, lr=args.lr, expert_state=prec)
    start = 0
    if args.resume:
        start = checkpoint.load(args.resume, model, trainer)
    batches = TokenBatches(cfg.vocab_size, args.seq, args.micro_batch, rank, world, args.seed, args.token_file,
                           args.token_dtype)

    def save_fn(path, step):
        checkpoint.save(path, model, trainer, step)

    # synthetic batches carry no label for their last position; file windows label every one
    valid = args.micro_batch * (args.seq if args.token_file else args.seq - 1)
    heartbeat = None
    if args.heartbeat_timeout > 0 and world > 1:
        from .utils.heartbeat import Heartbeat

        heartbeat = Heartbeat.from_default_group(timeout_s=args.heartbeat_timeout)
    timeline = None
    if args.stage_times:
        from .utils.trace import DeviceTimeline

        timeline = DeviceTimeline(capacity=64 * cfg.num_layers * 8, device=dev)
    train_loop(trainer, batches, args.steps, start, args.log_dir, args.ckpt_every, save_fn,
               ep if args.ep_stats else None, num_valid=valid, heartbeat=heartbeat, timeline=timeline)
    ep.check()
    ep.close()
    shutdown_comm()


if __name__ == "__main__":
    main()
