"""Placement planner (CPU): balance, replica tables, resharding over gloo."""
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spec_ep.parallel.placement import Placement, contiguous, loads_from_routing, plan_balanced, plan_from_routing, reshard


def _zipf_load(E, s, seed=0):
    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(E, generator=g) + 1
    return (1e6 * ranks.double() ** -s).round()


def test_contiguous_matches_reference_layout():
    p = contiguous(8, 4)
    assert p.owner == [0, 0, 1, 1, 2, 2, 3, 3]
    e2r, e2l, per = p.tables(1)
    assert e2r.tolist() == [0, 0, 1, 1, 2, 2, 3, 3]
    assert e2l.tolist() == [0, 1, 0, 1, 0, 1, 0, 1]
    assert per == [2, 2, 2, 2]


@pytest.mark.parametrize("s", [0.5, 1.0, 1.5])
def test_balanced_plan_reduces_imbalance(s):
    E, W = 128, 8
    load = _zipf_load(E, s)
    base = contiguous(E, W).imbalance(load)
    plan = plan_balanced(load, W)
    assert plan.imbalance(load) <= base + 1e-9
    assert sorted(e for r in plan.local_experts for e in r) == list(range(E))  # every expert once
    assert all(len(x) == E // W for x in plan.local_experts)
    # replicating the hottest experts to every rank helps further under heavy skew
    rep = plan_balanced(load, W, replicate_top=16)
    assert rep.imbalance(load) <= plan.imbalance(load) + 0.05
    if s >= 1.0:
        assert rep.imbalance(load) < base


def test_replica_tables_resolve_locally():
    E, W = 32, 4
    load = _zipf_load(E, 1.2)
    p = plan_balanced(load, W, replicate_top=4)
    for r in range(W):
        e2r, e2l, per = p.tables(r)
        assert per[r] == E // W + sum(1 for e in p.replicated if p.owner[e] != r)
        for e in range(E):
            d, slot = int(e2r[e]), int(e2l[e])
            assert p.local_experts[d][slot] == e
            if e in p.replicated:
                assert d == r  # served by this rank's own copy
            else:
                assert d == p.owner[e]
    assert Placement.from_dict(p.to_dict()) == p


def test_plan_from_routing_dump_format():
    L, T, K, E = 3, 64, 4, 16
    route = torch.randint(0, E, (L, T, K), dtype=torch.int16)
    loads = loads_from_routing(route, E)
    assert loads.shape == (L, E) and int(loads.sum()) == L * T * K
    plans = plan_from_routing(route, E, 4, replicate_top=2)
    assert len(plans) == L


def _reshard_worker(rank, world, init_file):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    E = 16
    old = contiguous(E, world)
    new = plan_balanced(_zipf_load(E, 1.0, seed=3), world, replicate_top=2)
    full = torch.arange(E * 6, dtype=torch.float32).view(E, 2, 3)
    w_old = full[old.local_experts[rank]]
    w_new = reshard(w_old, old, new)
    assert torch.equal(w_new, full[new.local_experts[rank]])
    dist.destroy_process_group()


def test_reshard_moves_weights(tmp_path: Path):
    mp.spawn(_reshard_worker, args=(4, tmp_path / "init"), nprocs=4)


def _replica_grad_worker(rank, port, out):
    import torch.distributed as dist

    from spec_ep.parallel.placement import plan_balanced
    from spec_ep.train import replica_slots, sum_replica_grads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        load = torch.tensor([50., 40, 3, 3, 2, 2, 1, 1])
        pl = plan_balanced(load, 2, replicate_top=2)
        slots = replica_slots(pl, rank)
        assert [pl.local_experts[rank][s] for s in slots] == sorted(pl.replicated)
        g = torch.full((pl.slots(rank), 3), float(rank + 1))
        for i, e in enumerate(pl.local_experts[rank]):
            g[i] *= e + 1
        before = g.clone()
        sum_replica_grads(g, slots)
        for i, e in enumerate(pl.local_experts[rank]):
            if e in pl.replicated:  # (1 + 2) * (e + 1): both copies' rows summed
                assert torch.equal(g[i], torch.full((3,), 3.0 * (e + 1)))
            else:
                assert torch.equal(g[i], before[i])
        out[rank] = True
    finally:
        dist.destroy_process_group()


def test_replicated_expert_gradients_are_summed_over_holders():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out = mp.Manager().dict()
    mp.spawn(_replica_grad_worker, args=(port, out), nprocs=2, join=True)
    assert out.get(0) and out.get(1)


def test_partial_replication_holders_tables_and_balance():
    g = torch.Generator().manual_seed(4)
    load = (torch.rand(16, generator=g) * 10) + torch.tensor([80.0, 60, 40] + [0.0] * 13)
    W = 4
    pl = plan_balanced(load, W, replicate_top=3, copies=2)
    assert sorted(pl.replicated) == [0, 1, 2]
    for e in range(16):
        hs = pl.holders_of(e)
        assert pl.owner[e] in hs and len(hs) == (2 if e in pl.replicated else 1)
        for r in hs:
            assert e in pl.local_experts[r]
    assert sorted(e for r in range(W) for e in pl.local_experts[r] if pl.owner[e] == r) == list(range(16))
    for src in range(W):
        e2r, e2l, _ = pl.tables(src)
        for e in range(16):
            d = int(e2r[e])
            assert d in pl.holders_of(e)
            if src in pl.holders_of(e):
                assert d == src
            assert pl.local_experts[d][int(e2l[e])] == e
    for e in pl.replicated:  # the sources without a copy split evenly over the holders
        hs = pl.holders_of(e)
        served = [pl.serving_rank(s, e) for s in range(W) if s not in hs]
        assert max(served.count(h) for h in hs) - min(served.count(h) for h in hs) <= 1
    assert pl.imbalance(load) <= plan_balanced(load, W).imbalance(load) + 1e-9
    back = Placement.from_dict(pl.to_dict())
    assert back.holders == pl.holders and back.tables(1)[0].tolist() == pl.tables(1)[0].tolist()


def _partial_worker(rank, port, out):
    import torch.distributed as dist

    from spec_ep.rbd import dedup_combine_dispatch
    from spec_ep.train import replica_slots, sum_replica_grads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=4)
    try:
        load = torch.tensor([90., 70, 50, 4, 3, 3, 2, 2, 2, 1, 1, 1, 1, 1, 1, 1])
        pl = plan_balanced(load, 4, replicate_top=3, copies=2)
        g = torch.Generator().manual_seed(50 + rank)
        T, k, H = 128, 3, 8
        logits = torch.randn(T, 16, generator=g) + torch.log(load)
        w, route = torch.softmax(logits, -1).topk(k, -1)
        x = torch.randn(T, H, generator=g)

        def fn(rows, ids):
            return torch.sin(rows * (ids.unsqueeze(-1) + 1.0))

        base = dedup_combine_dispatch(x, w, fn, route, 16)
        part = dedup_combine_dispatch(x, w, fn, route, 16, e2r=pl.tables(rank)[0])
        torch.testing.assert_close(part, base, rtol=1e-5, atol=1e-5)
        # gradients of partially replicated experts: summed over their holders only
        slots = replica_slots(pl, rank)
        grad = torch.full((pl.slots(rank), 2), float(rank + 1))
        sum_replica_grads(grad, slots)
        for i, e in enumerate(pl.local_experts[rank]):
            want = float(sum(h + 1 for h in pl.holders_of(e))) if e in pl.replicated else float(rank + 1)
            assert torch.equal(grad[i], torch.full((2,), want)), (rank, e, grad[i])
        out[rank] = True
    finally:
        dist.destroy_process_group()


def test_partial_replication_routing_and_gradients_gloo():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out = mp.Manager().dict()
    mp.spawn(_partial_worker, args=(port, out), nprocs=4, join=True)
    assert all(out.get(r) for r in range(4))
