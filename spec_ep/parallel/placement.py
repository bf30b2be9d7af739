"""Speculative expert placement: routing histograms -> expert-to-rank map + replica set.

The reference only sketches this idea (docs/plan.md:3-21: predict the hot experts, keep a
copy of every expert somewhere, replicate/shuffle experts for load balance). Here it is a
host planner whose output drives the dispatch kernels directly:

* Every expert has exactly one *primary* rank (so every expert exists somewhere).
* ``plan_balanced`` assigns primaries by greedy longest-processing-time bin packing of
  the measured per-expert loads, ``E / world`` slots per rank.
* ``replicate_top`` hot experts additionally get *replica* slots: on every rank by
  default (a token routed to a replicated expert is then served by its own rank's copy,
  no transfer at all), or with ``copies=c`` on ``c`` ranks only (the primary plus the
  ``c - 1`` least-loaded ranks). A source without a copy sends to one holder; the
  sources without a copy are dealt round-robin over the holders, so each holder serves
  an equal share of them.
* ``Placement.tables(rank)`` returns the per-rank ``(e2r, e2l)`` lookup tables the
  dispatch kernel uses: destination rank and local slot for each expert, as seen from
  that source rank.
* ``reshard`` moves expert weights between ranks when the placement changes.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class Placement:
    num_experts: int
    world: int
    owner: list[int]                      # primary rank of each expert
    local_experts: list[list[int]]        # per rank: global expert id of each local slot
    replicated: list[int] = field(default_factory=list)  # experts with more than one copy
    holders: dict[int, list[int]] | None = None  # ranks holding each replicated expert (None: every rank)

    # -----------------------------------------------------------------------------
    def holders_of(self, expert: int) -> list[int]:
        """Ranks holding a copy of ``expert`` (ascending)."""
        if expert not in self.replicated:
            return [self.owner[expert]]
        if self.holders is None or expert not in self.holders:
            return list(range(self.world))
        return sorted(self.holders[expert])

    def serving_rank(self, source: int, expert: int) -> int:
        """Rank whose copy of ``expert`` serves tokens of ``source``: its own copy if it
        holds one, else the holders in turn over the sources without a copy."""
        hs = self.holders_of(expert)
        if source in hs:
            return source
        if len(hs) == 1:
            return hs[0]
        others = [r for r in range(self.world) if r not in hs]
        return hs[others.index(source) % len(hs)]

    def slots(self, rank: int) -> int:
        return len(self.local_experts[rank])

    def per_rank(self) -> list[int]:
        return [len(x) for x in self.local_experts]

    def slot_of(self, rank: int, expert: int) -> int:
        return self.local_experts[rank].index(expert)

    def tables(self, rank: int) -> tuple[torch.Tensor, torch.Tensor, list[int]]:
        """(e2r, e2l, experts_per_rank) seen from source ``rank``.

        A replicated expert resolves to this rank's own copy when it holds one, else to
        ``serving_rank``; any other expert to its primary rank and the primary's slot.
        """
        E = self.num_experts
        e2r = torch.empty(E, dtype=torch.int32)
        e2l = torch.empty(E, dtype=torch.int32)
        rep = set(self.replicated)
        for e in range(E):
            d = self.serving_rank(rank, e) if e in rep else self.owner[e]
            e2r[e], e2l[e] = d, self.local_experts[d].index(e)
        return e2r, e2l, self.per_rank()

    def expected_rows(self, load: torch.Tensor, source_share: torch.Tensor | None = None) -> torch.Tensor:
        """Rows each rank computes for per-expert ``load`` (tokens routed to each expert).

        Replicated experts are served locally, so their load splits across ranks in the
        proportion ``source_share`` (uniform by default).
        """
        load = load.double()
        share = source_share.double() if source_share is not None else torch.full((self.world,), 1.0 / self.world,
                                                                                 dtype=torch.float64)
        rows = torch.zeros(self.world, dtype=torch.float64)
        rep = set(self.replicated)
        for e in range(self.num_experts):
            if e in rep:
                for src in range(self.world):
                    rows[self.serving_rank(src, e)] += load[e] * share[src]
            else:
                rows[self.owner[e]] += load[e]
        return rows

    def imbalance(self, load: torch.Tensor) -> float:
        rows = self.expected_rows(load)
        return float(rows.max() / rows.mean().clamp_min(1e-9))

    def to_dict(self) -> dict:
        d = {"num_experts": self.num_experts, "world": self.world, "owner": list(self.owner),
             "local_experts": [list(x) for x in self.local_experts], "replicated": list(self.replicated)}
        if self.holders is not None:
            d["holders"] = {str(e): list(h) for e, h in self.holders.items()}
        return d

    @staticmethod
    def from_dict(d: dict) -> "Placement":
        holders = d.get("holders")
        if holders is not None:
            holders = {int(e): list(h) for e, h in holders.items()}
        return Placement(d["num_experts"], d["world"], list(d["owner"]), [list(x) for x in d["local_experts"]],
                         list(d.get("replicated", [])), holders)


def contiguous(num_experts: int, world: int) -> Placement:
    """Expert e on rank e // (E / world) (the reference's fixed layout, src/rbd.py:200-202)."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    epr = num_experts // world
    owner = [e // epr for e in range(num_experts)]
    return Placement(num_experts, world, owner, [list(range(r * epr, (r + 1) * epr)) for r in range(world)])


def plan_balanced(load: torch.Tensor, world: int, replicate_top: int = 0, copies: int | None = None) -> Placement:
    """Greedy LPT packing of per-expert ``load`` onto ranks with E / world primary slots each,
    plus replicas of the ``replicate_top`` most loaded experts: on every rank, or with
    ``copies`` < world on that many ranks (see :func:`_partial_holders`).

    Replicated experts' load is spread evenly across ranks before packing the rest, since
    each source serves them locally; their primary copies are dealt round-robin so every
    rank keeps primary slots for the non-replicated experts.
    """
    E = load.numel()
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    if copies is not None and copies < world:
        if copies < 1:
            raise ValueError("copies must be at least 1")
        return _partial_holders(plan_balanced(load, world, 0), load, replicate_top, copies)
    cap = E // world
    load = load.double().cpu()
    order = torch.argsort(load, descending=True).tolist()
    replicated = sorted(order[:replicate_top])
    base = torch.zeros(world, dtype=torch.float64)
    for e in replicated:
        base += load[e] / world
    owner = [-1] * E
    slots = [[] for _ in range(world)]
    for i, e in enumerate(order[:replicate_top]):
        r = i % world
        while len(slots[r]) >= cap:  # more replicas than primary slots on this rank
            r = (r + 1) % world
        slots[r].append(e)
        owner[e] = r
    heap = [(float(base[r]), r) for r in range(world)]
    heapq.heapify(heap)
    for e in order[replicate_top:]:
        full = []
        while True:
            cur, r = heapq.heappop(heap)
            if len(slots[r]) < cap:
                break
            full.append((cur, r))
        slots[r].append(e)
        owner[e] = r
        add = 0.0 if e in replicated else float(load[e])
        heapq.heappush(heap, (cur + add, r))
        for item in full:
            heapq.heappush(heap, item)
    local = []
    for r in range(world):
        prim = sorted(slots[r])
        reps = [e for e in replicated if owner[e] != r]
        local.append(prim + reps)
    return Placement(E, world, owner, local, replicated)


def _partial_holders(base: Placement, load: torch.Tensor, replicate_top: int, copies: int) -> Placement:
    """Add ``copies - 1`` replicas of each of the ``replicate_top`` hottest experts to
    ``base`` (primaries unchanged). Experts are taken hottest first; each replica goes to
    the rank with the least expected rows at that point (ties: lowest rank), and the
    expected rows are recomputed with the expert's load split over its holders."""
    load = load.double().cpu()
    order = torch.argsort(load, descending=True).tolist()[:replicate_top]
    pl = Placement(base.num_experts, base.world, list(base.owner), [list(x) for x in base.local_experts], [], {})
    for e in order:
        hs = [pl.owner[e]]
        pl.replicated.append(e)
        pl.holders[e] = hs
        for _ in range(copies - 1):
            rows = pl.expected_rows(load)
            cand = [r for r in range(pl.world) if r not in hs]
            r = min(cand, key=lambda x: (float(rows[x]), x))
            hs.append(r)
            hs.sort()
            pl.local_experts[r].append(e)
    pl.replicated.sort()
    return pl


def loads_from_routing(route: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Per-layer expert loads from a ``[L, T, K]`` routing dump -> ``[L, E]``."""
    if route.dim() != 3:
        raise ValueError(f"routing dump must be [L, T, K], got shape {tuple(route.shape)}")
    if route.numel() and (int(route.min()) < 0 or int(route.max()) >= num_experts):
        raise ValueError("routing dump holds expert ids outside [0, num_experts)")
    L = route.shape[0]
    return torch.stack([torch.bincount(route[l].reshape(-1).long(), minlength=num_experts) for l in range(L)])


def plan_from_routing(route: torch.Tensor, num_experts: int, world: int, replicate_top: int = 0,
                      copies: int | None = None) -> list[Placement]:
    """One placement per layer from recorded routing (the experts_rank*.pt format)."""
    return [plan_balanced(l, world, replicate_top, copies) for l in loads_from_routing(route, num_experts)]


# ---------------------------------------------------------------------------------------
def gather_expert_rows(w_local: torch.Tensor, placement: Placement, rank: int, experts: list[int]) -> torch.Tensor:
    """Rows of ``w_local`` ([slots, ...]) holding the given global experts."""
    idx = [placement.slot_of(rank, e) for e in experts]
    return w_local[idx]


def reshard(w_local: torch.Tensor, old: Placement, new: Placement, group=None) -> torch.Tensor:
    """Move expert weights from ``old`` to ``new`` placement (collective over ``group``).

    Every slot of the new layout is filled from the old primary copy of its expert, over
    one variable-size all-to-all. Works on any backend (gloo for tests, NCCL on GPUs).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    per = w_local[0].numel()
    # what each rank needs, ordered by source (old primary)
    need = [[[] for _ in range(world)] for _ in range(world)]  # need[dst][src] = experts
    for dst in range(world):
        for e in new.local_experts[dst]:
            need[dst][old.owner[e]].append(e)
    send_rows = []
    send_counts = []
    for dst in range(world):
        es = need[dst][rank]
        send_counts.append(len(es) * per)
        if es:
            send_rows.append(gather_expert_rows(w_local, old, rank, es).reshape(-1))
    recv_counts = [len(need[rank][src]) * per for src in range(world)]
    send = torch.cat(send_rows) if send_rows else w_local.new_empty(0)
    recv = w_local.new_empty(sum(recv_counts))
    dist.all_to_all_single(recv, send.contiguous(), recv_counts, send_counts, group=group)
    got = {}
    off = 0
    for src in range(world):
        for e in need[rank][src]:
            got[e] = recv[off:off + per].view_as(w_local[0])
            off += per
    return torch.stack([got[e] for e in new.local_experts[rank]])
