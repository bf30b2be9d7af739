"""Fraction of roofline for the training step and the dispatch + combine layer.

Reads ``bench.py`` JSON lines (one per GPU count) or measured values given on the
command line, and prints, per row, the roofline bound (the slower of compute at the
measured bf16 peak, HBM bytes at the measured copy bandwidth and NVLink bytes at the
measured peer bandwidth), what bounds it, and measured time as a fraction of it.
Runs on the CPU.

    python benchmarks/roofline.py --bench out_1gpu.json out_8gpu.json
    python benchmarks/roofline.py --train 1:202.1:8bit 8:212.6:fp32 --dc 8:693
    python benchmarks/roofline.py ... --markdown          # table for the docs
"""
import argparse
import json
import os
import re
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from spec_ep.models.config import get_config  # noqa: E402
from spec_ep.utils.roofline import (Peaks, dispatch_combine_roofline, fraction,  # noqa: E402
                                    synthetic_layer_rows, train_step_roofline)

SEQ, HIDDEN, TOPK, EXPERTS = 4096, 2048, 8, 128


def from_bench(path):
    """(train rows, dispatch rows) from the JSON lines of a bench.py output file."""
    train, dc = [], []
    for line in open(path):
        line = line.strip()
        if not line.startswith("{"):
            continue
        d = json.loads(line)
        if d.get("impl", "spec_ep") != "spec_ep" or "ms_per_step" not in d:
            continue
        n = int(d["n_gpus"])
        m = re.search(r"experts: (\w+)", d.get("config", {}).get("optimizer", ""))
        train.append((n, float(d["ms_per_step"]), m.group(1) if m else "fp32"))
        if d.get("dispatch_combine_us_per_layer") is not None:
            dc.append((n, float(d["dispatch_combine_us_per_layer"]), None))
    return train, dc


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--bench", nargs="*", default=[], help="files with bench.py JSON lines")
    ap.add_argument("--train", nargs="*", default=[], help="N:ms_per_step:expert_state (8bit|fp32)")
    ap.add_argument("--dc", nargs="*", default=[],
                    help="N:us_per_layer[:rows_per_token]; rows default to the worst rank's max(sent, received) "
                         "on the benchmark's Zipf s=1.0 routing")
    ap.add_argument("--tokens", type=int, default=SEQ, help="tokens per rank of the --dc rows")
    ap.add_argument("--fp8", action="store_true", help="--dc rows dispatch e4m3 rows with 1x128 fp32 scales")
    ap.add_argument("--peaks", default=os.path.join(ROOT, "MEASURED_PEAKS.json"))
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--markdown", action="store_true")
    args = ap.parse_args()

    peaks = Peaks.load(args.peaks)
    cfg = get_config(args.model)
    train, dc = [], []
    for f in args.bench:
        t, d = from_bench(f)
        train += t
        dc += d
    for s in args.train:
        n, ms, state = s.split(":")
        train.append((int(n), float(ms), state))
    for s in args.dc:
        p = s.split(":")
        dc.append((int(p[0]), float(p[1]), float(p[2]) if len(p) > 2 else None))

    rows = []
    for n, ms, state in sorted(train):
        r = train_step_roofline(cfg, SEQ, SEQ, n, state, peaks)
        rows.append({"path": "training step", "n_gpus": n, "measured_ms": ms, "expert_state": state,
                     "compute_ms": r["compute_ms"], "hbm_ms": r["hbm_ms"], "nvlink_ms": r["nvlink_ms"],
                     "bound_ms": r["bound_ms"], "bound_by": r["bound_by"], "fraction": fraction(r["bound_ms"], ms)})
    for n, us, rpt in sorted(dc, key=lambda x: x[0]):
        if rpt is None:  # the slowest link: the rank that sends or receives the most rows
            rpt = synthetic_layer_rows(n, args.tokens, HIDDEN, EXPERTS, TOPK)["worst_rows_per_token"]
        r = dispatch_combine_roofline(args.tokens, HIDDEN, TOPK, rpt, peaks,
                                      HIDDEN + HIDDEN // 128 * 4 if args.fp8 else None)
        name = "dispatch+combine" + (" (fp8 dispatch)" if args.fp8 else "")
        rows.append({"path": name, "n_gpus": n, "measured_ms": us / 1e3, "remote_rows_per_token": rpt,
                     "compute_ms": 0.0, "hbm_ms": r["hbm_ms"], "nvlink_ms": r["nvlink_ms"],
                     "bound_ms": r["bound_ms"], "bound_by": r["bound_by"], "fraction": fraction(r["bound_ms"], us / 1e3)})

    if not args.markdown:
        for row in rows:
            print(json.dumps({**row, "peaks": peaks.source}))
        return
    print(f"Peaks ({peaks.source}): HBM {peaks.hbm_gbs:.0f} GB/s, bf16 {peaks.bf16_tflops_sustained:.0f} TFLOP/s "
          f"sustained, peer {peaks.peer_gbs:.0f} GB/s, all-reduce bus {peaks.allreduce_bus_gbs:.0f} GB/s\n")
    print("| path | GPUs | measured | compute | HBM | NVLink | bound by | fraction of roofline |")
    print("|---|---|---|---|---|---|---|---|")
    for row in rows:
        print(f"| {row['path']} | {row['n_gpus']} | {row['measured_ms']:.3f} ms | {row['compute_ms']:.3f} ms "
              f"| {row['hbm_ms']:.3f} ms | {row['nvlink_ms']:.3f} ms | {row['bound_by']} | {row['fraction']:.0%} |")


if __name__ == "__main__":
    main()
