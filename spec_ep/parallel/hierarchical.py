"""Two-stage hierarchical dispatch/combine over logical GPU groups (forward).

The reference's RBD (src/rbd.py:1-30, :417-506) moves tokens in two levels: one *pilot*
row per (token, other node) crosses nodes to the rank owning the token's first expert
on that node, which fans it out to the node's other experts; combine reverses it and
returns one merged row per (token, node). On one NVSwitch box the "nodes" become
logical groups of ``group_size`` ranks. This module builds that path from the fused
kernels:

  stage A  pilot transport (one row per (token, other group), dedup by pilot rank);
           each row carries the expert ids / weights of its choices in that group
  stage B  the regular fused EP dispatch -> experts -> combine, restricted to each
           group, over [own tokens ; received pilot rows] (the receive slab of stage A,
           so pilot rows are never copied)
  stage A' the pilot rows' group sums go back to their sources (combine of stage A),
           and the own-group sums are added in the source-side reduction.

Cross-group traffic is one row per (token, other group) each way; in-group traffic is
one row per (token or pilot row, rank). Forward only (benchmark path of the two-level
scheme; training uses the flat path).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import grouped_gemm as gg
from ..ops._ext import load
from .ep import ExpertParallel


class HierarchicalEP:
    def __init__(self, num_experts, top_k, hidden, max_tokens, group_size, placement=None, group=None,
                 timeout_s=10.0, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world % group_size:
            raise ValueError(f"world {self.world} is not a multiple of group_size {group_size}")
        self.gs, self.k, self.H, self.cap = group_size, top_k, hidden, max_tokens
        self.timeout_s = float(timeout_s)
        C = load()
        self.A = C.EpComm(self.world, self.rank, max_tokens, top_k, hidden, self.device.index or 0)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.A.ipc_handle(), group=group)
            self.A.open_peers(handles)
            dist.barrier(group=group)
        self.B = ExpertParallel(num_experts, top_k, hidden, self.world * max_tokens, group=group,
                                placement=placement, timeout_s=timeout_s, device=self.device)
        self.xs, self.es, self.ws = self.A.slabs()
        W, cap = self.world, max_tokens
        inv = torch.full((W, cap, top_k), -1, dtype=torch.int32, device=self.device)
        inv[:, :, 0] = torch.arange(W * cap, dtype=torch.int32, device=self.device).view(W, cap)
        self.inv_A = inv
        self.zero_w = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.epoch = 0
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.last_pilot_rows = None

    def check(self):
        self.B.check()
        code = int(self.status.item())
        if code:
            self.status.zero_()
            raise RuntimeError(f"hierarchical EP kernel error {code}")

    def close(self):
        self.B.close()
        self.A.close()

    def pilot_tables(self, topk_e):
        """Stage-A routing: pilot rank for choices in other groups, -1 for own group."""
        owner = self.B.e2r[topk_e.long()]
        grp = torch.div(owner, self.gs, rounding_mode="floor")
        mine = self.rank // self.gs
        first = (grp.unsqueeze(2) == grp.unsqueeze(1)).int().argmax(-1)  # first choice in the same group
        pilot = owner.gather(1, first)
        other = grp != mine
        dst = torch.where(other, pilot, -1).int().contiguous()
        meta = torch.where(other, topk_e.int(), -1).int().contiguous()  # expert ids ride with the pilot
        return dst, meta, other

    @torch.no_grad()
    def forward(self, x, topk_e, topk_w, w_gu=None, w_d=None):
        """MoE output for ``x`` [T, H]; identity experts when no weights are given."""
        T, H, W, cap, k, dev = x.shape[0], self.H, self.world, self.cap, self.k, self.device
        if T > cap:
            raise ValueError(f"{T} tokens exceed capacity {cap}")
        self.epoch += 1
        ep = self.epoch
        topk_w = topk_w.float().contiguous()
        dst_a, meta_a, other = self.pilot_tables(topk_e)
        slot_a = torch.empty(T, W, dtype=torch.int32, device=dev)
        send_a = torch.empty(W, dtype=torch.int32, device=dev)
        self_tok = torch.empty(cap, dtype=torch.int32, device=dev)
        rows_a = torch.empty(W, dtype=torch.int32, device=dev)
        self.A.route_plan(dst_a, slot_a, send_a)
        self.A.dispatch(x.contiguous(), dst_a, meta_a, topk_w, slot_a, self_tok, send_a, True, ep, self.done[0:1],
                        self.status, self.timeout_s, False)
        self.xs[self.rank, :T].copy_(x)  # own tokens join the stage-B token array in place
        self.A.wait_rows(send_a, rows_a, T, 0, ep, self.done[0:1], self.status, self.timeout_s)
        # stage-B routing over the slab: received pilot rows keep their expert ids, own
        # tokens keep their own-group choices, unused slots are masked out
        valid = torch.arange(cap, device=dev).unsqueeze(0) < rows_a.unsqueeze(1)  # [W, cap]
        e_b = torch.where(valid.unsqueeze(-1), self.es.int(), -1)
        e_b[self.rank] = -1
        e_b[self.rank, :T] = torch.where(other, -1, topk_e.int())
        w_b = self.ws.clone()
        w_b[self.rank, :T] = topk_w
        e_b = e_b.view(W * cap, k)
        st = self.B.dispatch_fwd(self.xs.view(W * cap, H), e_b, w_b.view(W * cap, k),
                                 tables=self.B.route_tables(e_b))
        if w_gu is None:
            y = st.xp
        else:
            h, _ = gg.gg_swiglu_fwd(st.xp, w_gu, st.group_off, status=self.status)
            y = gg.gg_fwd(h, w_d, st.group_off, status=self.status)
        out_b = self.B.combine_fwd(y, st)  # [W * cap, H] group sums of every B token
        self.A.combine(out_b, self.inv_A, self.zero_w, rows_a, False, None, T, ep, self.done[1:2], self.status,
                       self.timeout_s)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        own = out_b[self.rank * cap:self.rank * cap + T]
        self.A.source_reduce(slot_a, dst_a, own, out, None, ep, self.done[1:2], self.status, self.timeout_s)
        self.last_pilot_rows = send_a
        return out
