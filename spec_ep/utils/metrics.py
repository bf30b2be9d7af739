"""Structured per-rank metrics stream (JSON lines), aggregated on rank 0 with MAX over ranks."""
from __future__ import annotations

import json
import time
from pathlib import Path

import torch
import torch.distributed as dist


class MetricsWriter:
    def __init__(self, outdir, rank: int | None = None):
        self.rank = rank if rank is not None else (dist.get_rank() if dist.is_initialized() else 0)
        self.path = Path(outdir) / f"metrics_rank{self.rank}.jsonl"
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.f = open(self.path, "a")

    def log(self, step: int, **values):
        rec = {"ts": time.time(), "rank": self.rank, "step": step, **values}
        self.f.write(json.dumps(rec) + "\n")
        self.f.flush()

    def close(self):
        self.f.close()


def max_over_ranks(values: dict, device=None) -> dict:
    """Reduce scalar metrics with MAX over ranks (timings: the slowest rank decides)."""
    if not (dist.is_available() and dist.is_initialized()):
        return dict(values)
    keys = sorted(values)
    dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu")
    t = torch.tensor([float(values[k]) for k in keys], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return dict(zip(keys, t.tolist()))


def imbalance(tokens_per_rank: torch.Tensor) -> float:
    """max / mean of per-rank token counts (1.0 = perfectly balanced)."""
    t = tokens_per_rank.float()
    return float(t.max() / t.mean().clamp_min(1e-9))
