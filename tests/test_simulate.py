"""Host-side routing replay (spec_ep.parallel.simulate, benchmarks/replay_routing.py)."""
import os
import sys

import torch

from spec_ep.parallel.placement import contiguous, plan_balanced
from spec_ep.parallel.simulate import placement_traffic, replay_cache, split_steps, traffic

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_traffic_counts_by_hand():
    # 2 ranks, 4 experts (0,1 on rank 0; 2,3 on rank 1), top-2
    routes = [torch.tensor([[0, 1], [0, 2], [2, 3]]), torch.tensor([[3, 2], [0, 3]])]
    t = placement_traffic(routes, contiguous(4, 2))
    # rank 0 sends token 1 and token 2 to rank 1 (2 rows; naive 3 copies); rank 1 sends token 1 to rank 0
    assert t["remote_rows_per_token"] == 3 / 5 and t["naive_rows_per_token"] == 4 / 5
    assert t["recv_rows"] == [3.0, 4.0]
    # rank 0 sends 2 rows and receives 1, rank 1 the reverse: 2 rows per 2.5 tokens
    assert t["worst_link_rows_per_token"] == 2 / 2.5


def test_cache_replay_cuts_remote_rows_and_counts_fetches():
    g = torch.Generator().manual_seed(0)
    E, W, k = 32, 4, 4
    pop = torch.arange(E, 0, -1).float() ** 2
    steps = [[torch.multinomial(pop, 64 * k, replacement=True, generator=g).view(64, k) for _ in range(W)]
             for _ in range(6)]
    base = sum(traffic(s, [contiguous(E, W).tables(r)[0] for r in range(W)], W)["remote_rows_per_token"]
               for s in steps) / len(steps)
    oracle = replay_cache(steps, contiguous(E, W), slots=8, predict="oracle", expert_bytes=100, row_bytes=10)
    prev = replay_cache(steps, contiguous(E, W), slots=8, predict="previous", expert_bytes=100)
    assert oracle["mean_remote_rows_per_token"] < base and prev["mean_remote_rows_per_token"] < base
    assert oracle["fetched_bytes"] == 100 * oracle["fetches"] > 0
    assert prev["steps"][0]["fetches"] == 0  # nothing to predict the first step from
    assert 0.0 < prev["hit_rate"] <= 1.0
    # saved token bytes: (base - cached) remote rows, both directions, at row_bytes each
    want = sum((st["base_remote_rows_per_token"] - st["remote_rows_per_token"]) * W * 64 * 2 * 10
               for st in oracle["steps"])
    assert abs(oracle["saved_bytes"] - want) < 1e-6 and oracle["saved_bytes"] > 0
    assert prev["saved_bytes"] == 0.0  # row_bytes defaults to 0
    assert prev["steps"][0]["saved_bytes"] == 0.0
    # re-planning every 3 steps: fetches only on planning steps (1, 4 for "previous")
    sparse = replay_cache(steps, contiguous(E, W), slots=8, predict="previous", interval=3)
    assert all(st["fetches"] == 0 for st in sparse["steps"] if st["step"] not in (1, 4))
    assert sparse["fetches"] <= prev["fetches"]


def test_replay_cli_on_dumps(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    import replay_routing

    g = torch.Generator().manual_seed(1)
    files = []
    for r in range(4):
        d = torch.multinomial(torch.arange(16, 0, -1).float(), 2 * 256 * 2, replacement=True,
                              generator=g).view(2, 256, 2)
        files.append(str(tmp_path / f"experts_rank{r}.pt"))
        torch.save(d.to(torch.int16), files[-1])
    out = replay_routing.main(files + ["--num-experts", "16", "--top-k", "2", "--replicate-top", "2",
                                       "--slots", "2", "--tokens-per-step", "64"])
    schemes = {(o["layer"], o["scheme"]) for o in out}
    assert (1, "replicate_top2") in schemes and (0, "cache2_previous") in schemes and (0, "copies2_top2") in schemes
    assert all(o["remote_rows_per_token"] <= o["naive_rows_per_token"] + 1e-9 for o in out)
    assert split_steps([torch.zeros(2, 256, 2, dtype=torch.long)], 0, 64)[3][0].shape == (64, 2)
    assert plan_balanced(torch.ones(16), 4).imbalance(torch.ones(16)) == 1.0


def test_synthetic_drift_moves_the_hot_set():
    from spec_ep.utils.routing import synthetic_routing

    E = 32
    hot = []
    for b in (0, 1):
        _, te, _ = synthetic_routing(2048, 64, E, 4, s=1.5, seed=0, bias_seed=b)
        hot.append(set(torch.bincount(te.reshape(-1).long(), minlength=E).topk(4).indices.tolist()))
    assert hot[0] != hot[1]
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    import replay_routing

    out = replay_routing.main(["--synthetic", "--world", "2", "--num-experts", "16", "--top-k", "2", "--tokens", "256",
                               "--tokens-per-step", "64", "--drift-every", "2", "--hidden", "64", "--slots", "2",
                               "--replicate-top", "2", "--copies", "1"])
    cache = [o for o in out if o["scheme"] == "cache2_previous"]
    assert len(cache) == 1 and cache[0]["steps"] == 4 and "token_MiB_saved" in cache[0]
