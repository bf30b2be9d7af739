"""Roofline bounds (CPU): the closed forms against direct counts."""
import importlib.util
import json
import math
from pathlib import Path

import torch

from spec_ep.models.config import get_config
from spec_ep.utils.profile import FlopCounter
from spec_ep.utils.roofline import (Peaks, dispatch_combine_roofline, remote_ranks_uniform, synthetic_layer_rows,
                                    train_step_roofline)

ROOT = Path(__file__).resolve().parents[1]
PEAKS = Peaks(hbm_gbs=6500.0, bf16_tflops=1650.0, bf16_tflops_sustained=1400.0)


def test_remote_ranks_uniform_matches_sampling():
    assert remote_ranks_uniform(128, 8, 1) == 0.0
    assert abs(remote_ranks_uniform(128, 8, 8) - 7 * (1 - math.comb(112, 8) / math.comb(128, 8))) < 1e-12
    g = torch.Generator().manual_seed(0)
    T, E, k, W = 20000, 128, 8, 8
    e = torch.rand(T, E, generator=g).topk(k, -1).indices  # uniform k-subsets
    hot = torch.zeros(T, W, dtype=torch.bool).scatter_(1, e // (E // W), True)
    sampled = (hot.sum() - hot[:, 0].sum()).item() / T
    assert abs(sampled - remote_ranks_uniform(E, k, W)) < 0.03


def test_dispatch_combine_bytes():
    r = dispatch_combine_roofline(4096, 2048, 8, 1.0, PEAKS)
    assert r["nvlink_bytes"] == 4096 * 2048 * 2 * 2
    assert r["hbm_bytes"] == 2 * 4096 * 4096 + 2 * 4096 * 8 * 4096
    fp8 = dispatch_combine_roofline(4096, 2048, 8, 1.0, PEAKS, dispatch_row_bytes=2048 + 64)
    assert fp8["nvlink_bytes"] < r["nvlink_bytes"]
    assert dispatch_combine_roofline(4096, 2048, 8, 0.0, PEAKS)["bound_by"] == "hbm"


def test_train_step_bound_terms():
    cfg = get_config("qwen3-30b-a3b")
    one = train_step_roofline(cfg, 4096, 4096, 1, "8bit", PEAKS)
    assert one["flops"] == FlopCounter(cfg, 4096, 4096).step_flops(True)
    assert one["nvlink_ms"] == 0.0 and one["ep_bytes"] == 0.0
    assert abs(one["compute_ms"] - one["flops"] / 1.4e15 * 1e3) < 1e-9
    eight = train_step_roofline(cfg, 4096, 4096, 8, "8bit", PEAKS)
    assert eight["hbm_ms"] < one["hbm_ms"] and eight["nvlink_ms"] > 0
    assert eight["compute_ms"] == one["compute_ms"]  # weak scaling: same work per GPU
    assert train_step_roofline(cfg, 4096, 4096, 8, "fp32", PEAKS)["hbm_ms"] > eight["hbm_ms"]
    assert one["bound_ms"] == max(one["compute_ms"], one["hbm_ms"], one["nvlink_ms"])


def test_synthetic_layer_rows_conserve_rows():
    d = synthetic_layer_rows(4, tokens=512, hidden=64)
    assert sum(d["sent"]) == sum(d["received"])
    assert d["worst_rows_per_token"] >= d["mean_rows_per_token"] > 0
    assert max(d["sent"]) <= 3 * 512
    assert synthetic_layer_rows(1, tokens=64, hidden=16)["worst_rows_per_token"] == 0.0


def test_cli_reads_bench_lines(tmp_path, capsys, monkeypatch):
    spec = importlib.util.spec_from_file_location("roofline_cli", ROOT / "benchmarks" / "roofline.py")
    cli = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cli)
    line = {"metric": "m", "value": 1.0, "n_gpus": 1, "ms_per_step": 200.0, "impl": "spec_ep",
            "config": {"optimizer": "AdamW (dense: fp32 master+moments; experts: 8bit, updated in backward)"},
            "dispatch_combine_us_per_layer": 180.0}
    f = tmp_path / "bench.json"
    f.write_text("log line\n" + json.dumps(line) + "\n" + json.dumps({"impl": "reference", "unavailable": "x"}) + "\n")
    assert cli.from_bench(f) == ([(1, 200.0, "8bit")], [(1, 180.0, None)])
    monkeypatch.setattr("sys.argv", ["roofline.py", "--bench", str(f)])
    cli.main()
    rows = [json.loads(x) for x in capsys.readouterr().out.splitlines()]
    assert [r["path"] for r in rows] == ["training step", "dispatch+combine"]
    assert all(0 < r["fraction"] < 1 for r in rows)


def test_bench_fields_block():
    from spec_ep.utils.roofline import bench_fields

    cfg = get_config("qwen3-30b-a3b")
    out = bench_fields(cfg, 4096, 4096, 8, "fp32", 212.6, 693.0, ROOT / "MEASURED_PEAKS.json")
    assert out["training_step"]["bound_by"] in ("compute", "hbm", "nvlink")
    assert 0.2 < out["training_step"]["fraction"] < 0.5
    assert 0.3 < out["dispatch_combine"]["fraction"] < 0.6 and out["dispatch_combine"]["bound_by"] == "nvlink"
    json.dumps(out)  # goes into the benchmark's JSON line
    one = bench_fields(cfg, 4096, 4096, 1, "8bit", 202.1, None, None)
    assert one["peaks"] == "fallback" and "dispatch_combine" not in one
