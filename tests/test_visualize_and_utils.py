"""Routing dump format, visualiser (headless) and host-side utilities (CPU)."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_routing_recorder_dump_and_visualiser(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "visualization"))
    import visualize_expert_routing as viz

    from spec_ep.utils.profile import RoutingRecorder, load_routing

    for r in range(2):
        rec = RoutingRecorder()
        for l in range(3):
            rec.record(l, torch.randint(0, 16, (32, 4)))
        p = rec.save(tmp_path, rank=r)
        t = torch.load(p)
        assert t.dtype == torch.int16 and t.shape == (3, 32, 4)
    files = sorted(tmp_path.glob("experts_rank*.pt"))
    route = load_routing(files)
    assert route.shape == (3, 64, 4)
    out = viz.main([str(f) for f in files] + ["--num_experts", "16", "--num_gpus", "4"])
    assert out.exists() and out.stat().st_size > 0
    assert out.with_suffix(".csv").exists()


def test_flop_counter_matches_hand_count():
    from spec_ep.models.config import get_config
    from spec_ep.utils.profile import FlopCounter

    cfg = get_config("qwen3-30b-a3b")
    f = FlopCounter(cfg, 4096, 4096).forward_flops()
    # experts: 2 * T * k * 3 * H * I per layer
    assert f["experts_per_layer"] == 2 * 4096 * 8 * 3 * 2048 * 768
    assert f["total"] > 48 * f["experts_per_layer"]


def test_env_mapping_from_slurm(monkeypatch):
    from spec_ep.utils.dist import get_rank_and_world_size

    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setenv("SLURM_PROCID", "3")
    monkeypatch.setenv("SLURM_NTASKS", "8")
    monkeypatch.setenv("SLURM_LOCALID", "3")
    assert get_rank_and_world_size() == (3, 8)
    assert os.environ["LOCAL_RANK"] == "3"


def test_imbalance_metric():
    from spec_ep.utils.metrics import imbalance

    assert abs(imbalance(torch.tensor([10, 10, 10, 10])) - 1.0) < 1e-6
    assert abs(imbalance(torch.tensor([40, 0, 0, 0])) - 4.0) < 1e-6


def test_expert_transfer_group_splits():
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("expert_transfer", os.path.join(root, "benchmarks",
                                                                                  "expert_transfer.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    numel, world, gs = 6 * 64, 8, 4
    for balance in ("even", "uneven_internode", "uneven_intranode"):
        if balance == "uneven_internode":
            gs_b = 2  # four groups
        else:
            gs_b = gs
        sends, recvs = zip(*(mod.group_splits(numel, r, world, gs_b, balance, 0.5) for r in range(world)))
        for r in range(world):
            assert all(sends[r][d] == 0 for d in range(world) if d // gs_b == r // gs_b)  # nothing in-group
            for d in range(world):
                assert sends[r][d] == recvs[d][r]  # what r sends to d is what d expects from r
        if balance == "even":
            assert all(sum(s) == numel for s in sends)
        else:
            totals = sorted(sum(s) for s in sends)
            assert totals[0] == numel * 0.5 and totals[-1] == numel * 1.5
            assert sum(totals) == numel * world


def test_visualiser_counts_gpu_load_through_a_placement_with_replicas(tmp_path):
    import json

    sys.path.insert(0, os.path.join(ROOT, "visualization"))
    import visualize_expert_routing as viz

    from spec_ep.parallel.placement import plan_balanced

    E, W = 8, 2
    g = torch.Generator().manual_seed(0)
    dumps = [torch.randint(0, E, (2, 64, 2), generator=g) for _ in range(W)]
    dumps[0][..., 0] = 0  # expert 0 is hot
    load = torch.bincount(torch.cat(dumps, 1)[0].reshape(-1), minlength=E).float()
    pl = plan_balanced(load, W, replicate_top=1)
    files = []
    for r, d in enumerate(dumps):
        files.append(tmp_path / f"experts_rank{r}.pt")
        torch.save(d.to(torch.int16), files[-1])
    (tmp_path / "placement.json").write_text(json.dumps(pl.to_dict()))
    viz.main([str(f) for f in files] + ["--num_experts", str(E), "--num_gpus", str(W),
                                         "--placement", str(tmp_path / "placement.json")])
    rows = [line.split(",") for line in open(files[0].with_suffix(".csv")).read().splitlines()[1:]]
    gpu = {int(i): int(v) for l, kind, i, v in rows if kind == "gpu" and l == "0"}
    # each source's copies go where its own tables send them (expert 0 served locally)
    want = [0] * W
    for r, d in enumerate(dumps):
        for e in d[0].reshape(-1).tolist():
            want[int(pl.tables(r)[0][e])] += 1
    assert [gpu[i] for i in range(W)] == want
    assert sum(want) == 2 * 64 * 2 * W // 2


def test_flops_profile_file(tmp_path):
    from spec_ep.models.config import get_config
    from spec_ep.utils.profile import end_flops_profile, start_flops_profile

    class _M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.cfg = get_config("tiny")
            self.w = torch.nn.Parameter(torch.zeros(10))

    prof = start_flops_profile(_M(), tokens_per_rank=256, seq_len=256, training=True)
    path = end_flops_profile(prof, tmp_path)
    text = path.read_text()
    assert path.name == "flops_profile_0.txt"
    assert "experts (SwiGLU)" in text and "TFLOP/s" in text and "total" in text


def test_reference_import_paths_and_list_routing_hook():
    """``spec_ep.utils`` and ``spec_ep.utils_profile`` expose the reference's names
    (src/utils.py, src/utils_profile.py); the routing hook also fills a per-layer list as
    the reference's does."""
    from types import SimpleNamespace

    import spec_ep.utils as u
    import spec_ep.utils_profile as up

    for name in ("print0", "shutdown_comm", "get_rank_and_world_size"):
        assert callable(getattr(u, name))
    for name in ("count_params", "add_expert_statistics_hook", "report_peak_mem", "start_flops_profile",
                 "end_flops_profile", "torch_profile_ctx", "save_torch_profile"):
        assert callable(getattr(up, name))
    model = SimpleNamespace(layers=[SimpleNamespace(routing_callback=None) for _ in range(3)])
    sent = [None] * 3
    up.add_expert_statistics_hook(model, sent)
    for i, layer in enumerate(model.layers):
        layer.routing_callback(torch.full((4, 2), i + 5, dtype=torch.int32))
    assert all(s.dtype == torch.int16 and s.device.type == "cpu" and int(s[0, 0]) == i + 5
               for i, s in enumerate(sent))
