"""Roofline bounds for the fused paths: the slower of compute at the tensor-core peak,
bytes at the HBM copy bandwidth and bytes over NVLink at the peer-copy bandwidth.

Every bound is a lower bound on time from algorithmic work only (FLOPs of the model's
GEMMs and attention; the bytes that must be read or written at least once; the rows that
must cross NVLink under per-rank deduplication), so ``fraction = bound / measured`` is
at most about 1 for a kernel that does the work. The peaks come from a measured-peaks
JSON (``hbm_gbs``, ``bf16_tflops``, ``bf16_tflops_sustained``); NVLink figures are the
measured 8-rank all-reduce bus bandwidth (725 GB/s at 1 GiB) and peer copy (770 GB/s per
direction) of an 8xB200 NVSwitch system, overridable.

The reference measures only wall-clock latency of its MoE forward
(scripts/ds_moe.py:99-111) and GB/s of its all-to-alls
(benchmark/all2all/even_vs_uneven.py:36-73); it states no roofline.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

PEER_GBS = 770.0  # measured peer copy, GB/s per direction per GPU
ALLREDUCE_BUS_GBS = 725.0  # measured 8-rank NCCL all-reduce bus bandwidth at 1 GiB


@dataclass
class Peaks:
    hbm_gbs: float
    bf16_tflops: float  # burst: kernels timed in isolation
    bf16_tflops_sustained: float  # seconds-long loop under the power cap: kernels inside a long step
    peer_gbs: float = PEER_GBS
    allreduce_bus_gbs: float = ALLREDUCE_BUS_GBS
    source: str = "measured"

    @classmethod
    def load(cls, path: str | Path | None = None) -> "Peaks":
        """Peaks from a measured-peaks JSON; an earlier B200 measurement when absent."""
        if path is not None and Path(path).is_file():
            d = json.loads(Path(path).read_text())
            return cls(float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                       float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), source="measured")
        return cls(6650.0, 1590.0, 1400.0, source="fallback")


def remote_ranks_uniform(num_experts: int, top_k: int, world: int) -> float:
    """Expected other ranks a token reaches when its top-k is a uniform k-subset of the
    experts, laid out contiguously (E / world per rank): each other rank is missed with
    probability C(E - E/world, k) / C(E, k)."""
    if world <= 1:
        return 0.0
    per = num_experts // world
    miss = math.comb(num_experts - per, top_k) / math.comb(num_experts, top_k)
    return (world - 1) * (1.0 - miss)


def _bound(compute_ms: float, hbm_ms: float, link_ms: float) -> dict:
    parts = {"compute": compute_ms, "hbm": hbm_ms, "nvlink": link_ms}
    by = max(parts, key=parts.get)
    return {"compute_ms": compute_ms, "hbm_ms": hbm_ms, "nvlink_ms": link_ms, "bound_ms": parts[by], "bound_by": by}


# bytes of HBM traffic per parameter and step (minimum: each touched once per use)
EXPERT_BYTES = {
    # forward weight read 2 + dgrad weight read 2 + fused wgrad/AdamW epilogue (bf16 weight
    # read + write, two 8-bit moments read + written, block scales) 8.5
    "8bit": 12.5,
    # forward 2 + dgrad 2 + fp32 gradient written 4 + streaming AdamW (gradient 4, master,
    # m, v read + written 24, bf16 weight written 2) 34
    "fp32": 38.0,
}
# dense: forward + dgrad reads 4, bf16 gradient written and packed into its bucket 4,
# AdamW (gradient 2, fp32 master/m/v read + written 24, bf16 weight written 2) 28
DENSE_BYTES = 36.0


def train_step_roofline(cfg, tokens: int, seq_len: int, world: int, expert_state: str, peaks: Peaks,
                        remote_rows_per_token: float | None = None, replicas_per_rank: int = 0) -> dict:
    """Bound on one training step of a Qwen3-MoE-shaped model on one of ``world`` GPUs
    (weak scaling: ``tokens`` per GPU, experts sharded over the EP group).

    compute: analytic FLOPs (3x forward: QKV/O projections, causal attention, router,
      top-k SwiGLU experts, LM head) at the sustained bf16 peak.
    hbm: expert weights and optimizer state (``EXPERT_BYTES[expert_state]`` per local
      expert weight), dense weights and state (``DENSE_BYTES``), saved activations
      written once and read once (12 [T, H] tensors per layer plus the T*k expert rows of
      x and gate|up).
    nvlink: four row transfers per layer (forward dispatch and combine, backward dispatch
      of the output gradient and combine of the input gradient), ``remote_rows_per_token``
      rows of H bf16 each (default: uniform routing), plus the dense-gradient all-reduce
      (bf16) at the all-reduce bus bandwidth.
    """
    from .profile import FlopCounter

    H, I, L = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_layers
    flops = FlopCounter(cfg, tokens, seq_len).step_flops(training=True)
    compute_ms = flops / (peaks.bf16_tflops_sustained * 1e12) * 1e3
    total, expert = cfg.param_counts()
    dense = total - expert
    per_expert = 3 * H * I
    local_expert = expert / world + replicas_per_rank * L * per_expert
    act = L * (tokens * H * 2 * 12 + tokens * cfg.top_k * (H + 2 * I) * 2)
    hbm_bytes = EXPERT_BYTES[expert_state] * local_expert + DENSE_BYTES * dense + 2 * act
    hbm_ms = hbm_bytes / (peaks.hbm_gbs * 1e9) * 1e3
    if remote_rows_per_token is None:
        remote_rows_per_token = remote_ranks_uniform(cfg.num_experts, cfg.top_k, world)
    ep_bytes = 4 * L * remote_rows_per_token * tokens * H * 2
    ar_bytes = 2 * dense * 2 * (world - 1) / world if world > 1 else 0.0
    link_ms = (ep_bytes / (peaks.peer_gbs * 1e9) + ar_bytes / (peaks.allreduce_bus_gbs * 1e9)) * 1e3
    out = _bound(compute_ms, hbm_ms, link_ms)
    out.update(flops=flops, hbm_bytes=hbm_bytes, ep_bytes=ep_bytes, allreduce_bytes=ar_bytes,
               remote_rows_per_token=remote_rows_per_token)
    return out


def dispatch_combine_roofline(tokens: int, hidden: int, top_k: int, remote_rows_per_token: float, peaks: Peaks,
                              dispatch_row_bytes: int | None = None) -> dict:
    """Bound on one dispatch + combine of ``tokens`` rows (identity experts, no compute).

    nvlink: ``remote_rows_per_token`` rows out (``dispatch_row_bytes``, default bf16) and
      the same number of bf16 partials back, at the peer-copy bandwidth.
    hbm: the token rows read once, the ``tokens * top_k`` expert-ordered rows written
      once and read once by the combine, the output written once.
    """
    row = hidden * 2
    d_row = dispatch_row_bytes if dispatch_row_bytes is not None else row
    link_bytes = remote_rows_per_token * tokens * (d_row + row)
    hbm_bytes = 2 * tokens * row + 2 * tokens * top_k * row
    out = _bound(0.0, hbm_bytes / (peaks.hbm_gbs * 1e9) * 1e3, link_bytes / (peaks.peer_gbs * 1e9) * 1e3)
    out.update(nvlink_bytes=link_bytes, hbm_bytes=hbm_bytes)
    return out


def fraction(bound_ms: float, measured_ms: float) -> float:
    return bound_ms / measured_ms if measured_ms > 0 else float("nan")


def synthetic_layer_rows(world: int, tokens: int = 4096, hidden: int = 2048, num_experts: int = 128,
                         top_k: int = 8, s: float = 1.0, seed: int = 0) -> dict:
    """Rows that cross NVLink per rank for the dispatch benchmark's synthetic Zipf routing
    (contiguous placement, one row per (token, other rank)): per-rank rows sent and
    received, and the worst rank's max(sent, received) per token, which bounds the layer
    since every rank's ingress and egress are separate links of the same bandwidth."""
    import torch

    from .routing import synthetic_routing

    per = num_experts // world
    hits = []
    for r in range(world):
        _, te, _ = synthetic_routing(tokens, hidden, num_experts, top_k, s=s, seed=seed, rank=r)
        dst = torch.div(te.long(), per, rounding_mode="floor")
        hot = torch.zeros(tokens, world, dtype=torch.bool).scatter_(1, dst, True)
        hot[:, r] = False
        hits.append(hot.sum(0))  # rows rank r sends to each rank
    m = torch.stack(hits)  # [src, dst]
    sent, recv = m.sum(1).tolist(), m.sum(0).tolist()
    worst = max(max(a, b) for a, b in zip(sent, recv)) / tokens
    return {"sent": sent, "received": recv, "worst_rows_per_token": worst,
            "mean_rows_per_token": sum(sent) / (world * tokens)}


def bench_fields(cfg, tokens: int, seq_len: int, world: int, expert_state: str, step_ms: float,
                 dispatch_combine_us: float | None, peaks_path=None) -> dict:
    """Roofline block of the flagship benchmark's JSON line: the training step's bound and
    fraction, and the dispatch + combine layer's (worst rank's rows on the benchmark's
    Zipf s=1.0 routing, 4096 tokens/rank, hidden 2048, 128 experts, top-8)."""
    peaks = Peaks.load(peaks_path)

    def pick(r, measured_ms):
        return {"bound_ms": r["bound_ms"], "bound_by": r["bound_by"], "fraction": fraction(r["bound_ms"], measured_ms),
                "compute_ms": r["compute_ms"], "hbm_ms": r["hbm_ms"], "nvlink_ms": r["nvlink_ms"]}

    out = {"peaks": peaks.source,
           "training_step": pick(train_step_roofline(cfg, tokens, seq_len, world, expert_state, peaks), step_ms)}
    if dispatch_combine_us is not None:
        rows = synthetic_layer_rows(world)["worst_rows_per_token"]
        dc = dispatch_combine_roofline(4096, 2048, 8, rows, peaks)
        out["dispatch_combine"] = {**pick(dc, dispatch_combine_us / 1e3), "rows_per_token": rows}
    return out
