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
