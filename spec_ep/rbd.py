"""Redundancy-bypassing dispatch/combine (RBD) over ``torch.distributed``.

This module keeps the public API of the reference's ``spec_ep.rbd`` (src/rbd.py:38-506):
``InterPlan``, ``IntraPlan``, ``make_plan``, ``inter_node_dispatch``,
``intra_node_dispatch``, ``intra_node_combine``, ``merge_outputs``,
``inter_node_combine`` and ``RBD_combine_dispatch``, with the same plan semantics:

* A *copy* is one (token, expert) pair of ``route``.
* Copies whose expert lives on this rank's node go straight to the expert's rank.
* For every other node, the token's first copy on that node (route order) is the
  *pilot*; it crosses nodes once and its rank re-sends the token to the other experts
  of that node (the *replicas*, which include the pilot's own expert).
* Gate weights are applied by the rank that gathers a token's copies (the pilot rank
  for other-node copies, the source for same-node copies), so merged rows return
  already scaled.
* Output rows are in input token order; the expert callback sees rows in source-rank
  order with a parallel ``expert_ids`` tensor (src/rbd.py:454-455).

It runs on any backend (gloo on CPU, NCCL on GPU) and is the oracle the fused sm_100a
path (``spec_ep.parallel.ep``) is tested against. Two additions over the reference:

* Every all-to-all here is differentiable (the backward of a dispatch is the matching
  combine), so gradients reach tokens, gate weights and expert parameters
  (the reference notes "TODO: Support backprop", src/rbd.py:25-26).
* ``plan_traffic`` counts rows per stage, and ``dedup_combine_dispatch`` /
  ``naive_combine_dispatch`` implement the per-rank-dedup and plain per-copy
  all-to-all schemes used as byte-count baselines.
"""
from __future__ import annotations

from collections.abc import Callable
from typing import NamedTuple

import torch
import torch.distributed as dist


class InterPlan(NamedTuple):
    """Pilot traffic between nodes (src/rbd.py:38-51).

    pilot_token: [num_sent_pilots] token index of each pilot sent, in send order.
    pilot_send:  pilots sent to each global rank (0 for same-node ranks).
    pilot_recv:  pilots received from each global rank (0 for same-node ranks).
    """

    pilot_token: torch.Tensor
    pilot_send: list[int]
    pilot_recv: list[int]


class IntraPlan(NamedTuple):
    """Copy traffic inside a node, for local tokens or for received pilots (src/rbd.py:54-68).

    copy_row:    [num_copies] row each copy is taken from (token or pilot index).
    copy_weight: [num_copies] gate weight of each copy.
    send:        copies sent to each rank of the node (this rank included).
    recv:        copies received from each rank of the node (this rank included).
    """

    copy_row: torch.Tensor
    copy_weight: torch.Tensor
    send: list[int]
    recv: list[int]


# ----------------------------------------------------------------------------------------
# differentiable variable-size all-to-all
# ----------------------------------------------------------------------------------------
def _a2a_raw(rows: torch.Tensor, send: list[int], recv: list[int], group, async_op=False):
    out = rows.new_empty((sum(recv), *rows.shape[1:]))
    work = dist.all_to_all_single(out, rows.contiguous(), recv, send, group=group, async_op=async_op)
    return out, work


class _AllToAll(torch.autograd.Function):
    """Rows grouped by destination -> rows grouped by source; backward runs it in reverse."""

    @staticmethod
    def forward(ctx, rows, send, recv, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        out, _ = _a2a_raw(rows, send, recv, group)
        return out

    @staticmethod
    def backward(ctx, grad):
        g, _ = _a2a_raw(grad.contiguous(), ctx.recv, ctx.send, ctx.group)
        return g, None, None, None


class _PendingAllToAll:
    """Handle returned by the async stage functions: ``wait()`` completes the transfer.

    When autograd is recording, the transfer is run synchronously inside an autograd
    Function (so it has a backward); ``wait`` is then a no-op.
    """

    def __init__(self, work=None):
        self._work = work

    def wait(self):
        if self._work is not None:
            self._work.wait()
            self._work = None


def _needs_grad(t: torch.Tensor) -> bool:
    return torch.is_grad_enabled() and t.requires_grad


def _start_all2all(rows, send, recv, group=None):
    if _needs_grad(rows):
        return _AllToAll.apply(rows, send, recv, group), _PendingAllToAll()
    out, work = _a2a_raw(rows, send, recv, group, async_op=True)
    return out, _PendingAllToAll(work)


def _all2all(rows, send, recv, group=None):
    if _needs_grad(rows):
        return _AllToAll.apply(rows, send, recv, group)
    out, _ = _a2a_raw(rows, send, recv, group)
    return out


def _exchange_counts(counts: torch.Tensor, group=None) -> torch.Tensor:
    """counts[r, c] rows this rank sends to rank r in transfer c -> rows it receives."""
    out = torch.empty_like(counts)
    dist.all_to_all_single(out, counts.contiguous(), group=group)
    return out


def _block_starts(counts: torch.Tensor) -> torch.Tensor:
    """Exclusive prefix sum: where each rank's block starts in rank-grouped rows."""
    return torch.cumsum(counts, 0) - counts


def _group_by_local_rank(copy_row, copy_weight, copy_expert, experts_per_rank, gpus_per_node):
    """Stable grouping of copies by the node-local rank owning their expert (src/rbd.py:148-175)."""
    owner = torch.div(copy_expert, experts_per_rank, rounding_mode="floor") % gpus_per_node
    order = torch.sort(owner, stable=True).indices
    counts = torch.bincount(owner, minlength=gpus_per_node)
    return copy_row[order], copy_weight[order], copy_expert[order], counts


# the reference's names for the two plan helpers (src/rbd.py:136-175), same contracts
_start_offsets = _block_starts
_sort_copies = _group_by_local_rank


# ----------------------------------------------------------------------------------------
# planning
# ----------------------------------------------------------------------------------------
def make_plan(
    route: torch.Tensor,
    weights: torch.Tensor,
    E: int,
    gpus_per_node: int,
    local_group: dist.ProcessGroup,
) -> tuple[InterPlan, IntraPlan, IntraPlan, torch.Tensor]:
    """Build the RBD plan and tell the receivers what is coming (src/rbd.py:178-302).

    Collective over the global group and ``local_group``; moves no token rows.
    Experts are placed contiguously, ``E // world`` per rank, and ranks are numbered
    contiguously by node.

    Returns ``(inter, local, replica, expert_ids)`` where ``expert_ids`` lists the expert
    of every row this rank's experts will receive: local rows first, then replica rows.
    """
    world, rank = dist.get_world_size(), dist.get_rank()
    epr = E // world
    T, k = route.shape
    dev = route.device
    num_nodes = world // gpus_per_node
    my_node = rank // gpus_per_node

    expert = route.reshape(-1)
    token = torch.arange(T, device=dev).repeat_interleave(k)
    weight = weights.reshape(-1)
    dst_rank = torch.div(expert, epr, rounding_mode="floor")
    dst_node = torch.div(dst_rank, gpus_per_node, rounding_mode="floor")
    same_node = dst_node == my_node

    # ---- same-node copies: straight to their expert's rank ----
    local_row, local_w, local_e, local_send = _group_by_local_rank(
        token[same_node], weight[same_node], expert[same_node], epr, gpus_per_node
    )

    # ---- other-node copies: one pilot per (token, node), the first in route order ----
    node_tk = dst_node.view(T, k)
    same_as = node_tk.unsqueeze(2) == node_tk.unsqueeze(1)  # [T, k(j), k(j')]
    earlier = torch.ones(k, k, dtype=torch.bool, device=dev).tril(-1)  # j' < j
    is_first = ~(same_as & earlier).any(-1)  # no earlier copy on the same node
    first_j = same_as.int().argmax(-1)  # first j' on the same node (== j for pilots)
    remote = ~same_node
    pilot_mask = is_first.reshape(-1) & remote

    # flattened index of each remote copy's pilot copy
    pilot_flat_of_copy = (torch.arange(T, device=dev).unsqueeze(1) * k + first_j).reshape(-1)[remote]
    pilot_flat = torch.nonzero(pilot_mask).flatten()  # token-major order
    pilot_rank = dst_rank[pilot_flat]
    by_rank = torch.sort(pilot_rank, stable=True).indices
    pilot_token = token[pilot_flat][by_rank]
    pilot_send = torch.bincount(pilot_rank, minlength=world)

    # position of each pilot among the pilots sent to the same rank
    send_pos = torch.empty_like(by_rank)
    send_pos[by_rank] = torch.arange(by_rank.numel(), device=dev)
    pos_at_rank = send_pos - _block_starts(pilot_send)[pilot_rank]
    # map flattened copy index -> pilot ordinal (index into pilot_flat)
    ordinal = torch.full((T * k,), -1, dtype=torch.long, device=dev)
    ordinal[pilot_flat] = torch.arange(pilot_flat.numel(), device=dev)
    copy_pilot = ordinal[pilot_flat_of_copy]

    # every remote copy's (pilot position, expert, weight) goes to its pilot's rank
    meta_rank = pilot_rank[copy_pilot]
    meta_order = torch.sort(meta_rank, stable=True).indices
    meta_send = torch.bincount(meta_rank, minlength=world)
    meta_ids = torch.stack([pos_at_rank[copy_pilot], expert[remote]], 1)[meta_order]
    meta_w = weight[remote][meta_order]

    pilot_recv, meta_recv = _exchange_counts(torch.stack([pilot_send, meta_send], 1)).T
    ms, mr = meta_send.tolist(), meta_recv.tolist()
    got_ids, _ = _a2a_raw(meta_ids, ms, mr, None)
    got_w = _all2all(meta_w, ms, mr)  # differentiable when the weights need a gradient

    src = torch.arange(world, device=dev).repeat_interleave(meta_recv)
    got_pilot = got_ids[:, 0] + _block_starts(pilot_recv)[src]
    rep_row, rep_w, rep_e, rep_send = _group_by_local_rank(
        got_pilot, got_w, got_ids[:, 1], epr, gpus_per_node
    )

    local_recv, rep_recv = _exchange_counts(torch.stack([local_send, rep_send], 1), local_group).T.tolist()
    ls, rs = local_send.tolist(), rep_send.tolist()
    expert_ids = torch.cat(
        [_a2a_raw(local_e, ls, local_recv, local_group)[0], _a2a_raw(rep_e, rs, rep_recv, local_group)[0]]
    )

    inter = InterPlan(pilot_token, pilot_send.tolist(), pilot_recv.tolist())
    local = IntraPlan(local_row, local_w, ls, local_recv)
    replica = IntraPlan(rep_row, rep_w, rs, rep_recv)
    return inter, local, replica, expert_ids


# ----------------------------------------------------------------------------------------
# stages
# ----------------------------------------------------------------------------------------
def inter_node_dispatch(tokens: torch.Tensor, inter: InterPlan) -> torch.Tensor:
    """Send pilots to their ranks on other nodes (collective, global group; src/rbd.py:305-317)."""
    return _all2all(tokens[inter.pilot_token], inter.pilot_send, inter.pilot_recv)


def intra_node_dispatch(rows: torch.Tensor, plan: IntraPlan, local_group):
    """Start sending copies of ``rows`` to expert ranks of this node (src/rbd.py:320-342).

    Returns ``(expert_inputs, work)``; ``expert_inputs`` is valid after ``work.wait()``.
    """
    return _start_all2all(rows[plan.copy_row], plan.send, plan.recv, local_group)


def intra_node_combine(outputs: torch.Tensor, plan: IntraPlan, local_group):
    """Start returning expert outputs inside the node, reversing intra_node_dispatch."""
    return _start_all2all(outputs, plan.recv, plan.send, local_group)


def merge_outputs(copy_outputs: torch.Tensor, plan: IntraPlan, num_rows: int) -> torch.Tensor:
    """Scale each copy's output by its weight and sum per row (local; src/rbd.py:371-391)."""
    scaled = copy_outputs * plan.copy_weight.to(copy_outputs.dtype).unsqueeze(-1)
    merged = copy_outputs.new_zeros((num_rows, *copy_outputs.shape[1:]))
    return merged.index_add(0, plan.copy_row, scaled)


def inter_node_combine(merged: torch.Tensor, inter: InterPlan, num_tokens: int) -> torch.Tensor:
    """Return merged pilot rows to their sources and add them per token (src/rbd.py:394-414)."""
    back = _all2all(merged, inter.pilot_recv, inter.pilot_send)
    out = merged.new_zeros((num_tokens, *merged.shape[1:]))
    return out.index_add(0, inter.pilot_token, back)


def RBD_combine_dispatch(
    tokens: torch.Tensor,
    weights: torch.Tensor,
    expert: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
    route: torch.Tensor,
    E: int,
    gpus_per_node: int,
    local_group,
    concurrent: bool = False,
) -> torch.Tensor:
    """Dispatch tokens, run ``expert(rows, expert_ids)``, combine (src/rbd.py:417-506).

    Collective. ``concurrent=True`` overlaps the intra-node transfers with the inter-node
    ones. Differentiable with respect to ``tokens``, ``weights`` and whatever the expert
    callback closes over.
    """
    inter, local, replica, expert_ids = make_plan(route, weights, E, gpus_per_node, local_group)
    T = tokens.shape[0]

    local_in, lw = intra_node_dispatch(tokens, local, local_group)
    if not concurrent:
        lw.wait()
    pilots = inter_node_dispatch(tokens, inter)
    if concurrent:
        lw.wait()

    rep_in, rw = intra_node_dispatch(pilots, replica, local_group)
    rw.wait()

    out = expert(torch.cat([local_in, rep_in]), expert_ids)
    local_out, rep_out = out.split([local_in.shape[0], rep_in.shape[0]])

    rep_copies, rw = intra_node_combine(rep_out, replica, local_group)
    rw.wait()
    merged = merge_outputs(rep_copies, replica, pilots.shape[0])

    local_copies, lw = intra_node_combine(local_out, local, local_group)
    if not concurrent:
        lw.wait()
    remote = inter_node_combine(merged, inter, T)
    if concurrent:
        lw.wait()
    return merge_outputs(local_copies, local, T) + remote


# ----------------------------------------------------------------------------------------
# byte accounting and baseline schemes
# ----------------------------------------------------------------------------------------
def plan_traffic(route: torch.Tensor, E: int, world: int, rank: int, gpus_per_node: int) -> dict:
    """Rows this rank sends per scheme for ``route`` ([T, k] expert ids).

    * ``naive``: one row per (token, expert) whose expert is on another rank.
    * ``rank_dedup``: one row per (token, destination rank != this rank).
    * ``rbd_inter``: pilots crossing nodes (one per (token, other node)).
    * ``rbd_intra``: same-node copies to other ranks (RBD does not dedup these).
    """
    epr = E // world
    dst = torch.div(route, epr, rounding_mode="floor")
    T = route.shape[0]
    naive = int((dst != rank).sum())
    onehot = torch.zeros(T, world, dtype=torch.bool, device=route.device)
    onehot.scatter_(1, dst, True)
    rank_dedup = int(onehot.sum() - onehot[:, rank].sum())
    node = torch.div(dst, gpus_per_node, rounding_mode="floor")
    my_node = rank // gpus_per_node
    n_nodes = world // gpus_per_node
    node_hot = torch.zeros(T, n_nodes, dtype=torch.bool, device=route.device)
    node_hot.scatter_(1, node, True)
    rbd_inter = int(node_hot.sum() - node_hot[:, my_node].sum())
    rbd_intra = int(((node == my_node) & (dst != rank)).sum())
    return dict(naive=naive, rank_dedup=rank_dedup, rbd_inter=rbd_inter, rbd_intra=rbd_intra)


def naive_combine_dispatch(tokens, weights, expert, route, E, group=None):
    """Plain per-copy all-to-all (one row per (token, expert)); the byte-count baseline."""
    world = dist.get_world_size(group)
    epr = E // world
    T, k = route.shape
    flat_e = route.reshape(-1)
    tok = torch.arange(T, device=route.device).repeat_interleave(k)
    dst = torch.div(flat_e, epr, rounding_mode="floor")
    order = torch.sort(dst, stable=True).indices
    send = torch.bincount(dst, minlength=world)
    recv = _exchange_counts(send.unsqueeze(1), group).flatten()
    s, r = send.tolist(), recv.tolist()
    rows = _all2all(tokens[tok[order]], s, r, group)
    ids, _ = _a2a_raw(flat_e[order], s, r, group)
    out = _all2all(expert(rows, ids), r, s, group)
    w = weights.reshape(-1)[order].to(out.dtype).unsqueeze(-1)
    return tokens.new_zeros(tokens.shape).index_add(0, tok[order], out * w)


def dedup_combine_dispatch(tokens, weights, expert, route, E, group=None, e2r=None):
    """Per-rank dedup: one row per (token, destination rank), weights applied at the
    expert rank and one partial per (token, rank) returned. This is the semantics of the
    fused sm_100a dispatch/combine kernels.

    ``e2r`` ([E], optional) is this source rank's expert -> rank table (placement with
    replicas, or a speculative replica cache: a replicated expert resolves to a local
    copy); default: contiguous experts. ``expert(rows, ids)`` always receives global
    expert ids, so any rank holding a copy computes the same function.
    """
    world = dist.get_world_size(group)
    epr = E // world
    T, k = route.shape
    dev = route.device
    if e2r is None:
        dst = torch.div(route, epr, rounding_mode="floor")  # [T, k]
    else:
        dst = e2r.to(dev).long()[route]
    hot = torch.zeros(T, world, dtype=torch.bool, device=dev)
    hot.scatter_(1, dst, True)
    pairs = torch.nonzero(hot.T)  # (rank, token) sorted by rank then token
    d_rank, d_tok = pairs[:, 0], pairs[:, 1]
    send = torch.bincount(d_rank, minlength=world)
    recv = _exchange_counts(send.unsqueeze(1), group).flatten()
    s, r = send.tolist(), recv.tolist()
    rows = _all2all(tokens[d_tok], s, r, group)
    meta_e, _ = _a2a_raw(route[d_tok], s, r, group)  # [rows, k] experts of each row
    meta_d, _ = _a2a_raw(dst[d_tok], s, r, group)    # [rows, k] rank the source chose for each
    meta_w = _all2all(weights[d_tok], s, r, group)
    me = dist.get_rank(group)
    mine = meta_d == me  # [rows, k]
    ri, rj = torch.nonzero(mine, as_tuple=True)
    y = expert(rows[ri], meta_e[ri, rj])
    part = rows.new_zeros(rows.shape).index_add(0, ri, y * meta_w[ri, rj].unsqueeze(-1).to(y.dtype))
    back = _all2all(part, r, s, group)
    return tokens.new_zeros(tokens.shape).index_add(0, d_tok, back)
