"""Host-side replay of recorded routing through placements and the speculative cache.

Answers, for a routing dump (``experts_rank{r}.pt``, int16 ``[L, T, K]`` per source rank),
what a placement or a replica cache would do to the traffic, without a GPU:

* ``traffic(routes, tables)`` — rows each source sends (one per (token, other rank), the
  fused kernels' dedup) and the naive per-copy count, rows each rank receives, the
  receive imbalance (max / mean), and the worst rank's max(rows sent, rows received over
  NVLink) per token, which bounds the dispatch's link time.
* ``replay_cache(steps, placement, slots, ...)`` — runs each rank's speculative LRU cache
  (``policy_reference``, the host twin of the policy kernel) over a sequence of steps:
  the prediction for a step is the step's own routing (``"oracle"``) or the previous
  step's (``"previous"``), and the traffic is measured on the step's actual routing
  through the tables the cache produced. Reports hits, fetches, fetched weight bytes and
  the token bytes the cache kept off NVLink.

Reference parity: the reference feeds its recorded routing to an all-to-all timing
benchmark (benchmark/all2all/even_vs_uneven.py:76-92) and sketches the caching idea in
docs/plan.md:3-21; this module evaluates the planner and the cache on the same dumps.
"""
from __future__ import annotations

import torch

from .placement import Placement
from .speculative import ReplicaCache


def traffic(routes: list[torch.Tensor], tables: list[torch.Tensor], world: int) -> dict:
    """``routes[r]``: ``[T_r, K]`` expert ids of source rank r; ``tables[r]``: its ``[E]``
    expert -> rank table."""
    sent = naive = tokens = 0
    recv = torch.zeros(world, dtype=torch.float64)  # rows each rank receives, its own included
    remote_in = torch.zeros(world, dtype=torch.float64)  # rows each rank receives from other ranks
    out_rows = torch.zeros(world, dtype=torch.float64)  # rows each rank sends to other ranks
    for r, (route, e2r) in enumerate(zip(routes, tables)):
        T = route.shape[0]
        dst = e2r.long()[route.long()]
        hot = torch.zeros(T, world, dtype=torch.bool).scatter_(1, dst, True)
        per_rank = hot.sum(0).double()
        recv += per_rank
        remote = per_rank.clone()
        remote[r] = 0
        remote_in += remote
        out_rows[r] = remote.sum()
        sent += int(remote.sum())
        naive += int((dst != r).sum())
        tokens += T
    # the slowest link bounds a dispatch (and its combine): the rank that sends or
    # receives the most rows over NVLink, per token of that rank's share
    worst = float(torch.maximum(out_rows, remote_in).max()) * world / max(tokens, 1)
    return {"remote_rows_per_token": sent / max(tokens, 1), "naive_rows_per_token": naive / max(tokens, 1),
            "recv_rows": recv.tolist(), "recv_imbalance": float(recv.max() / recv.mean().clamp_min(1e-9)),
            "worst_link_rows_per_token": worst}


def placement_traffic(routes: list[torch.Tensor], placement: Placement) -> dict:
    return traffic(routes, [placement.tables(r)[0] for r in range(placement.world)], placement.world)


def replay_cache(steps: list[list[torch.Tensor]], placement: Placement, slots: int, min_count: int = 1,
                 predict: str = "previous", expert_bytes: int = 0, row_bytes: int = 0, interval: int = 1) -> dict:
    """``steps[s][r]``: ``[T, K]`` routing of source rank r at step s (one layer).

    ``saved_bytes``: token rows the cache kept off NVLink against ``placement`` alone,
    counted both ways (dispatch row out, combine partial back) at ``row_bytes`` each; set
    it beside ``fetched_bytes`` (weights moved in) to see whether the cache pays.
    ``interval``: re-plan the caches only every that many steps and keep their tables in
    between (``enable_speculation(..., interval=N)``); ``min_count``: cache only experts
    predicted for at least that many of a rank's tokens."""
    if interval < 1:
        raise ValueError("interval must be at least 1")
    if predict not in ("oracle", "previous"):
        raise ValueError("predict must be 'oracle' or 'previous'")
    W = placement.world
    caches = [ReplicaCache(placement, r, slots, min_count, device="cpu") for r in range(W)]
    per_step = []
    for s, routes in enumerate(steps):
        if predict == "previous" and s == 0:
            tables = [placement.tables(r)[0] for r in range(W)]  # nothing to predict from yet
            fetched = 0
        elif (s - (predict == "previous")) % interval:
            tables = [c.e2r for c in caches]  # between re-plans: the last tables stay in force
            fetched = 0
        else:
            src = routes if predict == "oracle" else steps[s - 1]
            before = [int(c.stats[1]) for c in caches]
            for c, pred in zip(caches, src):
                c.plan_host(pred)
            fetched = sum(int(c.stats[1]) - b for c, b in zip(caches, before))
            tables = [c.e2r for c in caches]
        t = traffic(routes, tables, W)
        base = traffic(routes, [placement.tables(r)[0] for r in range(W)], W)
        tokens = sum(int(r.shape[0]) for r in routes)
        saved = (base["remote_rows_per_token"] - t["remote_rows_per_token"]) * tokens * 2 * row_bytes
        t.update(step=s, fetches=fetched, fetched_bytes=fetched * expert_bytes,
                 base_remote_rows_per_token=base["remote_rows_per_token"], saved_bytes=saved)
        per_step.append(t)
    hits = sum(int(c.stats[0]) for c in caches)
    fetches = sum(int(c.stats[1]) for c in caches)
    n = max(len(per_step), 1)
    return {"steps": per_step, "hits": hits, "fetches": fetches, "hit_rate": hits / max(hits + fetches, 1),
            "fetched_bytes": fetches * expert_bytes, "saved_bytes": sum(p["saved_bytes"] for p in per_step),
            "mean_remote_rows_per_token": sum(p["remote_rows_per_token"] for p in per_step) / n,
            "mean_recv_imbalance": sum(p["recv_imbalance"] for p in per_step) / n}


def split_steps(dumps: list[torch.Tensor], layer: int, tokens_per_step: int) -> list[list[torch.Tensor]]:
    """Cut every rank's ``[L, T, K]`` dump of one layer into consecutive steps."""
    T = min(d.shape[1] for d in dumps)
    n = max(T // tokens_per_step, 1)
    return [[d[layer, i * tokens_per_step:(i + 1) * tokens_per_step].long() for d in dumps] for i in range(n)]
