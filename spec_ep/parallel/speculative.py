"""Speculative expert replication for expert-parallel inference.

The reference describes speculative expert parallelism as an idea only (docs/plan.md:3-21):
predict the experts a layer's tokens will pick by applying the router to earlier
activations, bring the predicted experts onto the GPU ahead of time, evict the others
least-recently-used first, and keep one copy of every expert that is never evicted. This
module builds it on the B200 data plane:

* ``ReplicaCache`` — per (layer, rank) state: ``S`` cache slots after the rank's ``P``
  pinned slots (primaries plus any static replicas of the placement). ``update(pred_e)``
  runs one single-block kernel that (1) counts the predicted rows per expert, (2) picks
  the want set: the ``S`` non-local experts with the most predicted rows (at least
  ``min_count``), (3) keeps wanted experts that are cached, assigns each missing one to
  the least recently used unwanted slot, and (4) writes this rank's routing tables so
  every cached expert is served by the local copy. No host sync.
* ``SpeculativeExperts`` — one MoE layer's expert weights in a symmetric (IPC) buffer,
  ``[P + S]`` slots per weight array; primaries are loaded once, cache slots are filled by
  a kernel that reads the primary rank's buffer with 16-byte peer loads over NVLink.
  ``speculate(x_prev, ...)`` runs prediction, policy and fetch on a side stream so the
  copy overlaps the layer's attention; ``tables()`` makes the current stream wait for it.
* ``policy_reference`` — the same policy in plain Python/torch, the oracle of the kernel
  and the host planner on machines without a GPU.
* ``enable_speculation(model, ...)`` switches a ``Qwen3MoeForCausalLM`` to speculative
  inference (forward only: a replica's weight gradient would have to be merged into its
  primary, which the training engine does not do, so training with it raises).

Prediction rule: before layer l's attention, layer l's router is applied to
``RMSNorm(x_in; post_norm_l)`` where ``x_in`` is the residual stream entering layer l (the
previous layer's output). The attention's residual update is the only term missing.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .placement import Placement


def _owner_tables(placement: Placement):
    owner = torch.tensor(placement.owner, dtype=torch.int32)
    owner_slot = torch.tensor([placement.local_experts[placement.owner[e]].index(e)
                               for e in range(placement.num_experts)], dtype=torch.int32)
    return owner, owner_slot


def policy_reference(pred_e, rank, P, min_count, base_e2r, base_e2l, owner, owner_slot, slot_expert, slot_stamp,
                     step):
    """Host version of the cache update (same ties and order as the kernel).

    Updates ``slot_expert``, ``slot_stamp`` and ``step`` in place and returns
    ``(e2r, e2l, fetch_rank, fetch_slot, stats)`` with stats = [hits, fetches, predicted
    rows of non-local experts, of them served locally after the update].
    """
    E, S = base_e2r.numel(), slot_expert.numel()
    ids = pred_e.reshape(-1).long()
    ids = ids[(ids >= 0) & (ids < E)]
    cnt = torch.bincount(ids, minlength=E).tolist()
    b_r = base_e2r.tolist()
    cand = [e for e in range(E) if b_r[e] != rank and cnt[e] >= min_count and cnt[e] > 0]
    cand.sort(key=lambda e: (-cnt[e], e))
    want = {e: i for i, e in enumerate(cand[:S])}
    se = slot_expert.tolist()
    ss = slot_stamp.tolist()
    cached = {e: s for s, e in enumerate(se) if 0 <= e < E}
    hit = [0 <= e < E and e in want for e in se]
    misses = sorted((e for e in want if e not in cached), key=lambda e: want[e])
    free = sorted((s for s in range(S) if not hit[s]), key=lambda s: (ss[s], s))
    now = int(step[0]) + 1
    fetch_rank = [-1] * S
    fetch_slot = [-1] * S
    fetches = 0
    for e, s in zip(misses, free):
        se[s] = e
        ss[s] = now
        fetch_rank[s] = int(owner[e])
        fetch_slot[s] = int(owner_slot[e])
        fetches += 1
    hits = 0
    for s in range(S):
        if fetch_rank[s] < 0 and hit[s]:
            ss[s] = now
            hits += 1
    e2r = base_e2r.clone()
    e2l = base_e2l.clone()
    for s, e in enumerate(se):
        if 0 <= e < E:
            e2r[e] = rank
            e2l[e] = P + s
    cand_rows = sum(cnt[e] for e in range(E) if b_r[e] != rank)
    local_rows = sum(cnt[e] for e in range(E) if b_r[e] != rank and int(e2r[e]) == rank)
    slot_expert.copy_(torch.tensor(se, dtype=slot_expert.dtype))
    slot_stamp.copy_(torch.tensor(ss, dtype=slot_stamp.dtype))
    step.fill_(now)
    as_t = lambda v: torch.tensor(v, dtype=torch.int32)  # noqa: E731
    return e2r, e2l, as_t(fetch_rank), as_t(fetch_slot), [hits, fetches, cand_rows, local_rows]


class ReplicaCache:
    """LRU cache of replicas of other ranks' experts for one (layer, rank).

    Args:
        placement: the pinned placement (primaries and static replicas).
        rank: this rank.
        num_slots: cache slots ``S`` (local expert slots ``P .. P+S-1``).
        min_count: fewest predicted rows that make an expert worth fetching.
    """

    def __init__(self, placement: Placement, rank: int, num_slots: int, min_count: int = 1, device="cuda"):
        if num_slots < 1:
            raise ValueError("a replica cache needs at least one slot")
        dev = torch.device(device)
        self.rank, self.S, self.min_count = int(rank), int(num_slots), int(min_count)
        self.P = placement.slots(rank)
        self.E = placement.num_experts
        e2r, e2l, _ = placement.tables(rank)
        owner, owner_slot = _owner_tables(placement)
        i32 = dict(dtype=torch.int32, device=dev)
        self.base_e2r, self.base_e2l = e2r.to(**i32), e2l.to(**i32)
        self.owner, self.owner_slot = owner.to(**i32), owner_slot.to(**i32)
        self.slot_expert = torch.full((self.S,), -1, **i32)
        self.slot_stamp = torch.full((self.S,), -1, **i32)
        self.step = torch.zeros(1, **i32)
        self.e2r, self.e2l = self.base_e2r.clone(), self.base_e2l.clone()
        self.fetch_rank = torch.full((self.S,), -1, **i32)
        self.fetch_slot = torch.full((self.S,), -1, **i32)
        self.stats = torch.zeros(4, dtype=torch.int64, device=dev)

    def update(self, pred_e: torch.Tensor):
        """Device update from predicted expert ids ``pred_e`` [T, k] (sm_100a kernel)."""
        from ..ops._ext import load

        load().spec_policy(pred_e.int().contiguous(), self.rank, self.P, self.min_count, self.base_e2r,
                           self.base_e2l, self.owner, self.owner_slot, self.slot_expert, self.slot_stamp, self.step,
                           self.e2r, self.e2l, self.fetch_rank, self.fetch_slot, self.stats)

    def plan_host(self, pred_e: torch.Tensor):
        """The same update computed on the host (planning without a GPU; kernel oracle)."""
        cpu = lambda t: t.detach().cpu()  # noqa: E731
        se, ss, st = cpu(self.slot_expert).clone(), cpu(self.slot_stamp).clone(), cpu(self.step).clone()
        e2r, e2l, fr, fs, stats = policy_reference(cpu(pred_e), self.rank, self.P, self.min_count, cpu(self.base_e2r),
                                                   cpu(self.base_e2l), cpu(self.owner), cpu(self.owner_slot), se, ss,
                                                   st)
        dev = self.e2r.device
        for dst, src in ((self.slot_expert, se), (self.slot_stamp, ss), (self.step, st), (self.e2r, e2r),
                         (self.e2l, e2l), (self.fetch_rank, fr), (self.fetch_slot, fs)):
            dst.copy_(src.to(dev))
        self.stats += torch.tensor(stats, dtype=torch.int64, device=dev)

    def summary(self) -> dict:
        """Accumulated hits / fetches and the share of predicted remote rows served locally."""
        h, f, cand, local = (int(v) for v in self.stats.tolist())
        return {"hits": h, "fetches": f, "hit_rate": h / max(h + f, 1), "predicted_remote_rows": cand,
                "predicted_rows_served_locally": local, "local_share": local / max(cand, 1)}


class MLPPredictor(torch.nn.Module):
    """The plan's second predictor (docs/plan.md:3-8): a small MLP on the residual stream
    that enters the layer (before attention), trained online to reproduce the layer's
    router choices. ``learn(x_in, topk_e)`` takes one Adam step of a multi-label loss
    (binary cross-entropy against the multi-hot of the chosen experts); ``predict``
    returns its top-k experts. Plain torch ops (GEMMs of [T, H] x [H, width]); the
    default predictor, the layer's own router on the residual stream, needs no training.
    """

    def __init__(self, hidden: int, num_experts: int, width: int = 256, lr: float = 1e-3, device=None,
                 dtype=torch.float32):
        super().__init__()
        self.net = torch.nn.Sequential(torch.nn.Linear(hidden, width), torch.nn.SiLU(),
                                       torch.nn.Linear(width, num_experts)).to(device=device, dtype=dtype)
        self.opt = torch.optim.Adam(self.net.parameters(), lr=lr)
        self.E = num_experts
        self.steps = 0

    def _in(self, x):
        x = x.to(self.net[0].weight.dtype)
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    @torch.no_grad()
    def predict(self, x_in: torch.Tensor, top_k: int) -> torch.Tensor:
        return self.net(self._in(x_in)).topk(top_k, -1).indices.int()

    def learn(self, x_in: torch.Tensor, topk_e: torch.Tensor) -> float:
        with torch.enable_grad():
            target = torch.zeros(x_in.shape[0], self.E, device=x_in.device, dtype=self.net[0].weight.dtype)
            target.scatter_(1, topk_e.long(), 1.0)
            loss = torch.nn.functional.binary_cross_entropy_with_logits(self.net(self._in(x_in.detach())), target)
            self.opt.zero_grad(set_to_none=True)
            loss.backward()
            self.opt.step()
        self.steps += 1
        return loss.detach()


class SpeculativeExperts:
    """One MoE layer's experts in a symmetric buffer with an LRU replica cache.

    Slot layout per weight array: ``[0, P)`` this rank's pinned experts (the copies peers
    read), ``[P, P + S)`` replicas of other ranks' experts. ``w_gu [P+S, 2I, H]`` and
    ``w_d [P+S, H, I]`` are views of the buffer, used directly by the grouped GEMMs.
    Collective construction over ``group``.
    """

    def __init__(self, placement: Placement, num_slots: int, hidden: int, inter: int, group=None, device=None,
                 min_count: int = 1, blocks_per_slot: int | None = None):
        from .symm import SymmetricBuffer

        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.cache = ReplicaCache(placement, self.rank, num_slots, min_count, self.device)
        self.P, self.S = self.cache.P, self.cache.S
        n = self.P + self.S
        # one layout on every rank (peers read each other's pinned slots at the same
        # offsets): sized for the rank with the most pinned slots
        self.p_max = max(placement.slots(r) for r in range(placement.world))
        n_layout = self.p_max + self.S
        self.gu_stride = 2 * inter * hidden * 2
        self.d_stride = hidden * inter * 2
        self.off_d = (n_layout * self.gu_stride + 255) // 256 * 256
        self.buf = SymmetricBuffer(self.off_d + n_layout * self.d_stride, group, self.device)
        self.w_gu = self.buf.view(torch.bfloat16, (n, 2 * inter, hidden), 0)
        self.w_d = self.buf.view(torch.bfloat16, (n, hidden, inter), self.off_d)
        # ~64 copy CTAs in total: enough loads in flight for NVLink, few SMs taken from attention
        self.blocks_per_slot = blocks_per_slot or max(1, 64 // self.S)
        self.stream = torch.cuda.Stream(device=self.device)
        self.ready = torch.cuda.Event()
        self.pending = False
        self.predictor: MLPPredictor | None = None
        self.interval = 1  # re-plan the cache every `interval` calls; reuse the tables between
        self.calls = 0
        self.planned = False  # this call re-planned the cache

    def observe(self, x_prev, topk_e):
        """Feed the layer's actual choices to its ``MLPPredictor`` (side stream), on the
        calls that re-planned the cache."""
        if self.predictor is None or not self.planned:
            return
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        x_prev.record_stream(self.stream)
        topk_e.record_stream(self.stream)
        with torch.cuda.stream(self.stream):
            self.predictor.learn(x_prev, topk_e)

    def load_primaries(self, w_gu: torch.Tensor, w_d: torch.Tensor):
        """Copy this rank's pinned experts in; collective (peers may read them afterwards)."""
        if w_gu.shape[0] != self.P or w_d.shape[0] != self.P:
            raise ValueError(f"expected {self.P} pinned experts, got {w_gu.shape[0]} / {w_d.shape[0]}")
        self.w_gu[:self.P].copy_(w_gu)
        self.w_d[:self.P].copy_(w_d)
        self.buf.barrier()

    def speculate(self, x_prev, post_norm, w_router, top_k, eps, renorm=True, bias=None, logit_bias=None):
        """Predict this layer's experts from ``x_prev`` (``predict_topk``, or the layer's
        ``MLPPredictor`` when one is set), update the cache and fetch the new replicas, all
        on the side stream after the work already queued on the current stream (so the
        fetch overlaps what the current stream runs next). Between re-plans (``interval``
        > 1) the call only counts and the cached tables stay in force."""
        self.planned = self.calls % self.interval == 0
        self.calls += 1
        if not self.planned:
            return
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        x_prev.record_stream(self.stream)  # read on the side stream: keep it allocated
        with torch.cuda.stream(self.stream):
            if self.predictor is not None:
                pred_e = self.predictor.predict(x_prev, top_k)
            else:
                pred_e = predict_topk(x_prev, post_norm, w_router, top_k, eps, renorm, bias, logit_bias)
            self.cache.update(pred_e)
            self.buf._b.fetch_experts(self.P, self.p_max, [0, self.off_d], [self.gu_stride, self.d_stride],
                                      self.cache.fetch_rank, self.cache.fetch_slot, self.blocks_per_slot)
        self.ready.record(self.stream)
        self.pending = True

    def tables(self):
        """(e2r, e2l) for this layer's dispatch; the current stream waits for the fetch."""
        if self.pending:
            torch.cuda.current_stream(self.device).wait_event(self.ready)
            self.pending = False
        return self.cache.e2r, self.cache.e2l

    def close(self):
        self.buf.close()


def predict_topk(x_prev, post_norm, w_router, top_k, eps, renorm=True, bias=None, logit_bias=None):
    """Predicted expert ids [T, k]: the layer's router on RMSNorm(x_prev; post_norm)."""
    from ..ops.linear import dense_fwd
    from ..ops.norm import rms_norm
    from ..ops.router import router_topk

    h = rms_norm(x_prev, post_norm, eps)
    logits = dense_fwd(h, w_router).float()  # the tcgen05 GEMM, on the caller's (side) stream
    if logit_bias is not None:
        logits = logits + logit_bias
    _, e = router_topk(logits, top_k, renorm, bias)
    return e


def enable_speculation(model, num_slots: int, min_count: int = 1, group=None, blocks_per_slot=None,
                       predictor: str = "router", predictor_width: int = 256, interval: int = 1):
    """Switch a ``Qwen3MoeForCausalLM`` to speculative expert replication (inference).

    Every layer's expert weights move into a ``SpeculativeExperts`` buffer (the layer's
    parameters become views of its pinned slots), and the shared ``ExpertParallel`` is
    widened to ``P + num_slots`` local expert groups. ``predictor`` is ``"router"`` (the
    layer's router on its incoming residual stream) or ``"mlp"`` (an ``MLPPredictor`` per
    layer, trained online from the routing it observes). ``interval`` > 1 re-plans each
    layer's cache only every that many calls (decode steps see a stable hot set; the
    prediction, policy and fetch launches then run once per ``interval`` steps).
    Collective over the EP group.
    """
    if interval < 1:
        raise ValueError("interval must be at least 1")
    if predictor not in ("router", "mlp"):
        raise ValueError("predictor must be 'router' or 'mlp'")
    ep = model.ep
    placement = ep.placement
    if placement is None:
        from .placement import contiguous

        placement = contiguous(ep.E, ep.world)
    cfg = model.cfg
    specs = []
    for layer in model.layers:
        sp = SpeculativeExperts(placement, num_slots, cfg.hidden_size, cfg.moe_intermediate_size,
                                group=group if group is not None else ep.group, device=ep.device,
                                min_count=min_count, blocks_per_slot=blocks_per_slot)
        sp.load_primaries(layer.w_gu.data, layer.w_d.data)
        layer.w_gu.data = sp.w_gu[:sp.P]
        layer.w_d.data = sp.w_d[:sp.P]
        if predictor == "mlp":
            sp.predictor = MLPPredictor(cfg.hidden_size, cfg.num_experts, predictor_width, device=ep.device)
        sp.interval = int(interval)
        layer.spec = sp
        specs.append(sp)
    ep.set_local_slots(specs[0].P + num_slots)
    return specs


def speculation_summary(model) -> dict:
    """Cache statistics summed over the layers of a model with speculation enabled."""
    tot = torch.zeros(4, dtype=torch.int64)
    for layer in model.layers:
        if getattr(layer, "spec", None) is not None:
            tot += layer.spec.cache.stats.cpu()
    h, f, cand, local = (int(v) for v in tot.tolist())
    return {"hits": h, "fetches": f, "hit_rate": h / max(h + f, 1), "predicted_remote_rows": cand,
            "local_share": local / max(cand, 1)}
