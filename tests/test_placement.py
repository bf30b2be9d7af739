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
