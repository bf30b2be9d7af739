"""Two-stage path, host side (CPU): the pilot tables follow the reference's pilot rule
(src/rbd.py:238-252): one pilot per (token, other group), the token's first choice in
that group in route order, sent to that choice's expert rank; choices in the token's own
group take no pilot."""
from types import SimpleNamespace

import pytest
import torch

from spec_ep.parallel.hierarchical import HierarchicalEP
from spec_ep.parallel.placement import contiguous, plan_balanced


def _oracle(topk_e, e2r, gs, rank):
    T, k = topk_e.shape
    dst = torch.full((T, k), -1, dtype=torch.int32)
    meta = torch.full((T, k), -1, dtype=torch.int32)
    mine = rank // gs
    for t in range(T):
        pilot_of_group = {}
        for j in range(k):
            e = int(topk_e[t, j])
            r = int(e2r[e])
            g = r // gs
            if g == mine:
                continue
            pilot_of_group.setdefault(g, r)  # first choice in route order
            dst[t, j] = pilot_of_group[g]
            meta[t, j] = e
    return dst, meta


@pytest.mark.parametrize("world,gs,balanced", [(8, 4, False), (8, 2, True), (4, 2, False)])
def test_pilot_tables_follow_the_rbd_pilot_rule(world, gs, balanced):
    E, k, T = 32, 4, 200
    g = torch.Generator().manual_seed(world * 10 + gs)
    topk_e = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    pl = plan_balanced(torch.rand(E, generator=g) * 10, world) if balanced else contiguous(E, world)
    for rank in range(world):
        e2r = pl.tables(rank)[0].long()
        stub = SimpleNamespace(B=SimpleNamespace(e2r=e2r), gs=gs, rank=rank)
        dst, meta, other = HierarchicalEP.pilot_tables(stub, topk_e)
        want_dst, want_meta = _oracle(topk_e, e2r, gs, rank)
        assert torch.equal(dst, want_dst) and torch.equal(meta, want_meta)
        assert torch.equal(other, want_dst >= 0)
        # one pilot rank per (token, other group): all of a group's choices share it
        grp = torch.div(e2r[topk_e], gs, rounding_mode="floor")
        for t in range(0, T, 17):
            for gg in set(grp[t].tolist()) - {rank // gs}:
                assert len(set(dst[t][grp[t] == gg].tolist())) == 1
