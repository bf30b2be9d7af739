"""Fused expert-parallel MoE over NVLink peer memory (one process per GPU).

Forward of one MoE layer on rank r (all on the device, no host sync):

  route_plan   slot[t][d]: ordinal of token t among the tokens r sends to rank d
  dispatch     one row per (token, destination rank) stored into the peer's slab,
               plus the row's (local expert, gate weight) choices; epoch header
  recv_plan    wait for every source's header, count rows per local expert,
               place each (row, choice) at a deterministic position of its expert group
               (64-row aligned, zero padding) and copy the rows (HBM fan-out)
  gate_up      tcgen05 grouped GEMM + SwiGLU epilogue  -> h, and gu saved for backward
  down         tcgen05 grouped GEMM                    -> y
  combine      gate-weighted sum of a token's co-resident experts, ONE partial row
               per (token, rank) stored back into the source's slab
  source_reduce  sum of the <= W partials per token in rank order (deterministic)

Backward mirrors it: dy is dispatched to the same slots, gathered into expert order,
then the fused down-dgrad + SwiGLU-backward GEMM (which also produces the router-weight
gradient and w*h), the two weight-gradient GEMMs, the gate_up dgrad, and a combine of
dx plus the router-weight gradients back to the sources.

Reference parity: this is the B200 version of ``RBD_combine_dispatch``
(src/rbd.py:417-506) with per-rank rather than per-node dedup (one NVSwitch domain);
the torch reference of the same semantics is ``spec_ep.rbd.dedup_combine_dispatch``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import grouped_gemm as gg
from ..ops._ext import load
from ..utils.profile import stage

GRAPH_EPOCH_BASE = 1 << 31  # epochs of graph-replayed calls: base + device counter

ERRORS = {1: "pipeline barrier timeout", 2: "peer rank never signalled (timeout)", 3: "receive capacity overflow",
          4: "bad argument", 5: "received row names an out-of-range local expert (corrupted metadata)"}


class EPError(RuntimeError):
    pass


def contiguous_placement(num_experts: int, world: int):
    """Expert e lives on rank e // (E / world) in local slot e % (E / world) (src/rbd.py:200-202)."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    epr = num_experts // world
    e = torch.arange(num_experts)
    return (e // epr).int(), (e % epr).int(), [epr] * world


@dataclass
class EPState:
    """Per-layer plan saved from forward for backward (all device tensors)."""

    T: int
    slot: torch.Tensor
    send_count: torch.Tensor
    self_tok: torch.Tensor
    dst_tk: torch.Tensor   # destination rank of each (token, choice); -1 = not sent
    meta_tk: torch.Tensor  # local expert slot on that rank
    topk_w: torch.Tensor
    rows_from: torch.Tensor
    group_off: torch.Tensor
    group_cnt: torch.Tensor
    xp: torch.Tensor
    row_w: torch.Tensor
    row_src: torch.Tensor
    inv_rows: torch.Tensor
    local_bwd: tuple | None = None  # world size 1: (input-gradient rows, router-weight grads) for the finish


class ExpertParallel:
    """Communicator + plan for one expert-parallel group.

    Args:
        num_experts: experts of the layer (E).
        top_k: experts per token.
        hidden: model width (H).
        max_tokens: most tokens a rank passes in one call (sizes the symmetric slabs).
        group: process group of the EP ranks (None = default group, or single GPU).
        placement: a ``Placement`` from ``spec_ep.parallel.placement`` (or raw
            ``(e2r, e2l, experts_per_rank)`` tables); default: contiguous experts.
        capacity_factor: unused (kept for API compatibility): buffers are sized exactly per
            call from the device-side row count.
        timeout_s: device-side wait limit before a peer is declared lost.
        fp8_dispatch: send forward-pass rows to other ranks as e4m3 with one fp32 scale
            per 128 values (2,112 instead of 4,096 bytes per 2048-wide row); backward
            traffic stays bf16.
    """

    def __init__(self, num_experts, top_k, hidden, max_tokens, group=None, placement=None,
                 capacity_factor=2.0, timeout_s=10.0, device=None, fp8_dispatch=False):
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.E, self.k, self.H, self.cap = num_experts, top_k, hidden, max_tokens
        if placement is None:
            placement = contiguous_placement(num_experts, self.world)
        if hasattr(placement, "tables"):  # a spec_ep.parallel.placement.Placement
            self.placement = placement
            e2r, e2l, per_rank = placement.tables(self.rank)
        else:
            self.placement = None
            e2r, e2l, per_rank = placement
        self.e2r = e2r.to(self.device, torch.int32)
        self.e2l = e2l.to(self.device, torch.int32)
        self.G = int(per_rank[self.rank])
        C = load()
        self.comm = C.EpComm(self.world, self.rank, max_tokens, top_k, hidden, self.device.index or 0)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.comm.ipc_handle(), group=group)
            self.comm.open_peers(handles)
            dist.barrier(group=group)
        # worst case: every token of every source routes all k choices here
        self.cap_rows = self.world * max_tokens * top_k + self.G * 64
        self.timeout_s = float(timeout_s)
        self.epoch = 0
        self.cur_epoch = 0
        self.epoch_dev = None  # device epoch counter, set by graph_epochs(True)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.fp8_dispatch = bool(fp8_dispatch)
        if self.fp8_dispatch and hidden % 128:
            raise ValueError("fp8 dispatch needs hidden % 128 == 0")
        self.stats_on = False  # traffic statistics of forward dispatches (enable_stats)
        self._reset_stats()
        # row budget of a pass (begin_pass / end_pass): receive buffers sized ahead of the
        # device-side count, so no layer waits for a device->host read
        self._budget = 0       # rows every call of a pass may receive (0: not learned yet)
        self._seen = 0         # most rows a call needed in exact-size calls of this pass
        self._pass = None
        self._need = torch.zeros(1024, dtype=torch.int32, device=self.device)
        self._miss = torch.zeros(1, dtype=torch.int32, device=self.device)

    # -------------------------------------------------------------------------------
    def _reset_stats(self):
        self.stat_sent = torch.zeros(self.world, dtype=torch.int64, device=self.device)
        self.stat_copies = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.stat_tokens = 0
        self.stat_recv_rows: list[int] = []

    def enable_stats(self, on: bool = True):
        """Accumulate forward-dispatch traffic on the device (two small reductions per
        layer call while on): rows sent per destination, remote (token, expert) copies,
        tokens, and the received row counts the host already reads."""
        self.stats_on = bool(on)

    def take_stats(self) -> dict:
        """Per-token traffic since the last call, then reset: ``remote_rows_per_token``
        (one row per (token, other rank), what the kernels send), ``naive_rows_per_token``
        (one row per remote (token, expert) copy, a plain all-to-all), and the mean
        received rows per layer call on this rank."""
        sent = self.stat_sent.tolist()
        copies = int(self.stat_copies.item())
        T = max(self.stat_tokens, 1)
        remote = sum(sent) - sent[self.rank]
        recv = self.stat_recv_rows
        out = {"remote_rows_per_token": remote / T, "naive_rows_per_token": copies / T,
               "recv_rows_per_call": (sum(recv) / len(recv)) if recv else 0.0, "tokens": self.stat_tokens}
        self._reset_stats()
        return out

    # -------------------------------------------------------------------------------
    def check(self):
        """Raise if any kernel recorded an error (one small device->host read)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            raise EPError(f"expert-parallel kernel error {code}: {ERRORS.get(code, 'unknown')}")

    def close(self):
        self.comm.close()

    def graph_epochs(self, on: bool = True):
        """Switch to (or from) a device-side epoch counter.

        Kernels validate peer headers against the epoch of their call. A captured CUDA
        graph replays its kernels with the arguments of the capture, so for capture each
        layer call instead bumps a device counter that every kernel of the call adds to a
        fixed base (2^31 and up, disjoint from the host-counted epochs). Every rank of the
        group must switch at the same call.
        """
        if on:
            if self.epoch_dev is None:
                self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.comm.set_device_epoch(self.epoch_dev)
        else:
            self.comm.set_device_epoch(None)
        self._graph = bool(on)

    def _next_epoch(self) -> int:
        if getattr(self, "_graph", False):
            self.epoch_dev.add_(1)
            self.cur_epoch = GRAPH_EPOCH_BASE
        else:
            self.epoch += 1
            self.cur_epoch = self.epoch
        return self.cur_epoch

    # -------------------------------------------------------------------------------
    # Row budgets: no host sync inside a pass
    # -------------------------------------------------------------------------------
    # One budget serves every call of a pass: the most rows any call has needed x margin
    # (64-row steps, at most the worst case cap_rows); after an overflow, the most rows a
    # call needed x growth. Routing drifts while a model trains (without a load-balancing
    # loss a rank's share of the choices can grow step after step) and a rank's received
    # rows vary from layer to layer; a budget per layer would be overflowed by one of
    # dozens of layers x ranks nearly every step. A miss costs a second forward, the
    # margin only memory (the saved expert activations of every layer).
    budget_margin = 1.5
    budget_growth = 2.0

    def begin_pass(self):
        """Start a pass of layer calls (e.g. one model forward). Inside a pass every
        ``dispatch_fwd`` sizes its receive buffers (and so every saved activation of its
        layer) from the learned row budget instead of reading the received row count back
        to the host, so the host never waits on the device between layers. The first
        pass learns the budget with exact sizes. A call whose rows exceed the budget
        empties its layout and raises a device flag; ``end_pass`` reports it and the
        caller runs the pass again, with the budget grown to fit."""
        self._pass = 0
        self._seen = 0

    def _grow_budget(self, rows: int, factor: float):
        want = min(self.cap_rows, (int(rows * factor) + 64 + 63) // 64 * 64)
        self._budget = max(self._budget, want)

    def run_pass(self, fn, retries: int = 3):
        """``fn()`` (e.g. one model forward) inside a pass, run again while some layer's
        rows outgrow their budget; returns its result. Collective over the default group
        when ranks run together (every rank must call it)."""
        for _ in range(retries + 1):
            self.begin_pass()
            out = fn()
            if not self.end_pass():
                return out
            del out
        raise EPError("MoE receive-row budgets kept overflowing")

    def end_pass(self) -> bool:
        """Close the pass; True if some call overflowed its budget (on any rank of the
        default process group) and the pass must be run again. One small device->host
        read (after a MAX all-reduce of the flag when ranks run together)."""
        n, self._pass = self._pass, None
        if not n:
            return False
        if self._seen:  # exact-size calls in this pass: learn the budget from them
            self._grow_budget(self._seen, self.budget_margin)
            self._seen = 0
        flag = self._miss.clone()
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        vals = torch.cat([flag, self._need[:n]]).tolist()
        self._miss.zero_()
        missed, need = bool(vals[0]), vals[1:]
        if self.stats_on:
            self.stat_recv_rows.extend(need)
        if missed:
            self._grow_budget(max(need), self.budget_growth)
        return missed

    def set_local_slots(self, G: int):
        """Number of local expert groups the receive side lays out (primaries plus, with
        speculative replication, the replica cache slots)."""
        self.G = int(G)
        self.cap_rows = self.world * self.cap * self.k + self.G * 64

    def route_tables(self, topk_e, e2r=None, e2l=None):
        """(dst_tk, meta_tk) for expert ids ``topk_e`` ([T, k]; negative ids are not sent),
        through this communicator's placement or the given ``(e2r, e2l)`` device tables."""
        e = topk_e.int().contiguous()
        dst = torch.empty_like(e)
        meta = torch.empty_like(e)
        self.comm.route_tables(e, self.e2r if e2r is None else e2r, self.e2l if e2l is None else e2l, dst, meta)
        return dst, meta

    def dispatch_fwd(self, x, topk_e, topk_w, tables=None, static_rows=False) -> EPState:
        """Send rows, build the expert-grouped receive layout. ``tables`` optionally gives
        precomputed ``(dst_tk, meta_tk)`` (e.g. the hierarchical path's pilot routing).

        ``static_rows`` sizes the receive buffers at their worst case instead of reading
        the received row count back to the host: no host sync, so the layer can be
        captured in a CUDA graph (inference; the expert GEMMs skip the unused rows).
        """
        T = x.shape[0]
        if T > self.cap:
            raise ValueError(f"{T} tokens exceed the communicator capacity {self.cap}")
        ep = self._next_epoch()
        idx = self._pass
        budget = 0
        if idx is not None and not static_rows and idx < self._need.numel():
            budget = self._budget
        rows_mode = -1 if static_rows else budget
        dst_in, meta_in = tables if tables is not None else (None, None)
        # one host call: tables, route plan, dispatch, receive count + scan, buffers sized
        # by the budget (no host read), the worst case, or an exact read, permute + gather
        (slot, send_count, self_tok, rows_from, group_off, group_cnt, xp, row_w, row_src, inv_rows, dst_tk, meta_tk,
         topk_w), R = self.comm.dispatch_forward(
            x, topk_e.int().contiguous(), topk_w, self.e2r, self.e2l, dst_in, meta_in, self.G, ep, rows_mode,
            self.cap_rows, self._need[idx:idx + 1] if budget else None, self._miss if budget else None,
            self.done[0:1], self.status, self.timeout_s, self.fp8_dispatch)
        if not static_rows and not budget and idx is not None:
            self._seen = max(self._seen, R)
        if idx is not None:
            self._pass = idx + 1
        if self.stats_on:
            self.stat_sent += send_count
            self.stat_copies += ((dst_tk >= 0) & (dst_tk != self.rank)).sum()
            self.stat_tokens += T
            if not static_rows and not budget:
                self.stat_recv_rows.append(R)
        return EPState(T, slot, send_count, self_tok, dst_tk, meta_tk, topk_w, rows_from, group_off, group_cnt, xp,
                       row_w, row_src, inv_rows)

    def combine_fwd(self, y, st: EPState, residual=None):
        return self.comm.combine_forward(y, st.inv_rows, st.row_w, st.rows_from, st.slot, st.dst_tk, residual, st.T,
                                         self.cur_epoch, self.done[1:2], self.status, self.timeout_s)

    def dispatch_bwd(self, dy, st: EPState):
        ep = self._next_epoch()
        if self.world > 1:  # at world size 1 the gather reads dy's rows in place
            self.comm.dispatch(dy, st.dst_tk, st.meta_tk, st.topk_w, st.slot, st.self_tok, st.send_count,
                               False, ep, self.done[0:1], self.status, self.timeout_s, False)
        dyp = torch.empty(st.xp.shape[0], self.H, dtype=torch.bfloat16, device=self.device)
        self.comm.recv_gather(dy, st.self_tok, st.row_src, st.group_off, st.send_count, dyp, ep, self.done[0:1],
                              self.status, self.timeout_s)
        return dyp

    def combine_bwd(self, dxp, row_dw, st: EPState):
        self.combine_bwd_send(dxp, row_dw, st)
        return self.combine_bwd_finish(st)

    def combine_bwd_send(self, dxp, row_dw, st: EPState):
        """Store this rank's input-gradient partials (and router-weight gradients) into the
        source ranks' return slabs; independent local work can run before the finish. At
        world size 1 nothing leaves the GPU: the finish does both steps in one kernel."""
        if self.world == 1:
            st.local_bwd = (dxp, row_dw)
            return
        self.comm.combine(dxp, st.inv_rows, st.row_w, st.rows_from, False, row_dw, st.T, self.cur_epoch,
                          self.done[1:2], self.status, self.timeout_s)

    def combine_bwd_finish(self, st: EPState):
        """Wait for every rank's partials of this layer and sum them per token."""
        dx = torch.empty(st.T, self.H, dtype=torch.bfloat16, device=self.device)
        dw = torch.empty(st.T, self.k, dtype=torch.float32, device=self.device)
        if self.world == 1:
            dxp, row_dw = st.local_bwd
            st.local_bwd = None
            self.comm.combine_local(dxp, st.inv_rows, st.row_w, st.slot, st.dst_tk, False, row_dw, None, dx, dw,
                                    self.status)
            return dx, dw
        self.comm.source_reduce(st.slot, st.dst_tk, None, dx, dw, self.cur_epoch, self.done[1:2],
                                self.status, self.timeout_s)
        return dx, dw


class EPGraph:
    """A callable that runs expert-parallel inference layers, captured as one CUDA graph.

    ``fn`` must size its layers without a host read, with ``dispatch_fwd(...,
    static_rows=True)`` (worst case) or inside a pass with a learned row budget, and read
    its inputs from tensors that stay allocated; copy new inputs into them and
    ``replay()``.
    Capture switches ``ep`` to device-side epochs (each replayed layer call bumps the
    counter on the device), runs ``warmup`` eager calls on a side stream, then captures
    one call. Every rank of the group must build and replay its graph in the same order.
    Errors recorded by the kernels surface through ``ep.check()`` as usual.
    """

    def __init__(self, ep: "ExpertParallel", fn, warmup: int = 2):
        self.ep, self.fn = ep, fn
        ep.graph_epochs(True)
        side = torch.cuda.Stream(device=ep.device)
        side.wait_stream(torch.cuda.current_stream(ep.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream(ep.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn()

    def replay(self):
        self.graph.replay()
        return self.out


class _EPMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, topk_w, w_gu, w_d, topk_e, ep: ExpertParallel, grad_sink, residual, route):
        with stage("ep.dispatch"):
            tables = ep.route_tables(topk_e, *route) if route is not None else None
            st = ep.dispatch_fwd(x.contiguous(), topk_e, topk_w, tables=tables)
        with stage("ep.experts"):
            h, gu = gg.gg_swiglu_fwd(st.xp, w_gu, st.group_off, status=ep.status)
            y = gg.gg_fwd(h, w_d, st.group_off, status=ep.status)
        del h
        with stage("ep.combine"):
            out = ep.combine_fwd(y, st, residual)
        ctx.ep, ctx.st, ctx.sink = ep, st, grad_sink
        ctx.has_residual = residual is not None
        ctx.save_for_backward(w_gu, w_d, gu)
        return out

    @staticmethod
    def backward(ctx, dout):
        ep, st, sink = ctx.ep, ctx.st, ctx.sink
        w_gu, w_d, gu = ctx.saved_tensors
        dout = dout.contiguous()
        with stage("ep.dispatch_bwd"):
            dyp = ep.dispatch_bwd(dout, st)
        row_dw = torch.zeros(st.xp.shape[0], dtype=torch.float32, device=dout.device)
        dgu, hw, row_dw = gg.gg_swiglu_bwd(dyp, w_d, st.group_off, gu, st.row_w, row_dw=row_dw, status=ep.status)
        dxp = gg.gg_dgrad(dgu, w_gu, st.group_off, status=ep.status)
        with stage("ep.combine_bwd"):
            ep.combine_bwd_send(dxp, row_dw, st)
        del dxp
        # The expert weight gradients (and their optimizer updates) feed nothing downstream,
        # so they run while the other ranks' partials of this layer are still in flight.
        fused = getattr(sink, "fused_wgrad", None) if sink is not None else None
        g_gu = g_d = None
        with stage("ep.expert_wgrad"):
            if fused is not None:  # optimizer applied inside the wgrad GEMM epilogue
                fused(w_d, dyp, hw, st.group_off, ep.status)
                fused(w_gu, dgu, st.xp, st.group_off, ep.status)
            else:
                dwd = gg.gg_wgrad(dyp, hw, st.group_off, ep.G, status=ep.status)
                dwgu = gg.gg_wgrad(dgu, st.xp, st.group_off, ep.G, status=ep.status)
                if sink is not None:
                    sink(w_d, dwd)
                    sink(w_gu, dwgu)
                else:
                    g_d = dwd.to(w_d.dtype) if ctx.needs_input_grad[3] else None
                    g_gu = dwgu.to(w_gu.dtype) if ctx.needs_input_grad[2] else None
        del hw, dyp, dgu
        with stage("ep.combine_bwd"):
            dx, dtopk_w = ep.combine_bwd_finish(st)
        ctx.st = None
        dres = dout if ctx.has_residual else None
        return dx, dtopk_w, g_gu, g_d, None, None, None, dres, None


def ep_moe(x, topk_e, topk_w, w_gu, w_d, ep: ExpertParallel, grad_sink=None, residual=None, route=None):
    """Expert-parallel SwiGLU MoE: ``out[t] = residual[t] + sum_j w[t,j] * FFN_{e[t,j]}(x[t])``.

    ``w_gu [G, 2I, H]`` and ``w_d [G, H, I]`` hold this rank's ``G`` local experts.
    ``grad_sink(param, fp32_grad)``, when given, receives the expert weight gradients
    (e.g. an optimizer applying them immediately) instead of autograd. ``route``
    optionally gives per-call ``(e2r, e2l)`` device tables (speculative replicas)
    instead of the communicator's placement.
    """
    return _EPMoE.apply(x, topk_w, w_gu, w_d, topk_e, ep, grad_sink, residual, route)
