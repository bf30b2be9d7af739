"""Profiling and statistics helpers (reference: src/utils_profile.py:11-74).

* ``count_params`` - total vs expert parameters.
* ``RoutingRecorder`` / ``add_expert_statistics_hook`` - capture each MoE layer's top-k
  expert ids (int16, on the host) and save them as ``experts_rank{r}.pt`` of shape
  [L, T, K], the format the visualiser and the placement planner read.
* ``report_peak_mem`` - per-rank peak allocated/reserved memory, printed in rank order.
* ``torch_profile_ctx`` / ``save_torch_profile`` - torch.profiler with CPU+CUDA activity,
  shapes, memory and FLOPs; Chrome trace per rank plus a key-averages table.
* ``FlopCounter`` - analytic FLOPs of one step of the MoE model (replaces DeepSpeed's
  FlopsProfiler, which is not available here) and achieved TFLOP/s.
* ``stage`` / ``enable_stage_ranges`` - NVTX ranges (also visible as labels in
  torch.profiler traces) around the expert-parallel stages; off by default, or with
  ``SEPX_NVTX=1`` in the environment, so a normal step pays nothing for them.
"""
from __future__ import annotations

import contextlib
import os
from pathlib import Path

import torch
import torch.distributed as dist
from torch.profiler import ProfilerActivity, profile, record_function  # noqa: F401


def _rank():
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _world():
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def count_params(module) -> tuple[int, int]:
    """(total, expert) parameter counts; expert = parameter names containing "expert" or
    flagged as expert weights."""
    total = sum(p.numel() for p in module.parameters())
    expert = sum(p.numel() for n, p in module.named_parameters()
                 if "expert" in n or getattr(p, "_sepx_expert", False))
    return total, expert


class RoutingRecorder:
    """Collects the top-k expert ids chosen in every MoE layer of a forward pass."""

    def __init__(self):
        self.layers: dict[int, torch.Tensor] = {}

    def record(self, layer_idx: int, topk_e: torch.Tensor):
        self.layers[layer_idx] = topk_e.detach().to(torch.int16).cpu()

    def stacked(self) -> torch.Tensor:
        return torch.stack([self.layers[i] for i in sorted(self.layers)])  # [L, T, K]

    def save(self, outdir, rank: int | None = None) -> Path:
        rank = _rank() if rank is None else rank
        path = Path(outdir) / f"experts_rank{rank}.pt"
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(self.stacked(), path)
        return path


def add_expert_statistics_hook(model, recorder):
    """Record the routing of every MoE layer of a ``spec_ep`` model; returns the layers
    hooked. ``recorder`` is a :class:`RoutingRecorder`, or, as in the reference
    (src/utils_profile.py:16-26), any container indexed by layer (``sent[i]`` receives
    that layer's int16 ``[T, K]`` expert ids on the host after each forward)."""
    handles = []
    for i, layer in enumerate(getattr(model, "layers", [])):
        if isinstance(recorder, RoutingRecorder):
            layer.routing_callback = (lambda e, i=i: recorder.record(i, e))
        else:
            def store(e, i=i):
                recorder[i] = e.detach().to(torch.int16).cpu()

            layer.routing_callback = store
        handles.append(layer)
    return handles


def load_routing(files) -> torch.Tensor:
    """Concatenate ``experts_rank*.pt`` dumps along the token dimension -> [L, T_total, K]."""
    return torch.cat([torch.load(f).long() for f in files], dim=1)


def report_peak_mem(device=None):
    """Print every rank's peak allocated / reserved GiB in rank order (barrier-serialised)."""
    dev = device if device is not None else torch.cuda.current_device()
    alloc = torch.cuda.max_memory_allocated(dev) / 2**30
    resv = torch.cuda.max_memory_reserved(dev) / 2**30
    for i in range(_world()):
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
        if i == _rank():
            print(f"rank {i}: peak allocated {alloc:.2f} GiB, peak reserved {resv:.2f} GiB", flush=True)
    return alloc, resv


def torch_profile_ctx(with_stack: bool = False):
    return profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True,
                   profile_memory=True, with_stack=with_stack, with_flops=True)


def save_torch_profile(prof, outdir, verbose: bool = False) -> Path:
    outdir = Path(outdir) / "profile"
    outdir.mkdir(parents=True, exist_ok=True)
    trace = outdir / f"trace_rank{_rank()}.json"
    prof.export_chrome_trace(str(trace))
    if verbose and _rank() == 0:
        (outdir / "key_averages.txt").write_text(
            prof.key_averages().table(sort_by="cuda_time_total", row_limit=30))
    return trace


class FlopCounter:
    """Analytic FLOPs of one training (or forward-only) step of a Qwen3-MoE-shaped model."""

    def __init__(self, cfg, tokens_per_rank: int, seq_len: int):
        self.cfg, self.T, self.S = cfg, tokens_per_rank, seq_len

    def forward_flops(self) -> dict:
        c, T = self.cfg, self.T
        H, D = c.hidden_size, c.head_dim
        qkv = 2 * T * H * c.qkv_width
        o = 2 * T * c.num_heads * D * H
        # causal attention: QK^T and PV over the lower triangle incl. diagonal
        pairs = (T // self.S) * self.S * (self.S + 1) // 2
        attn = 4 * pairs * D * c.num_heads
        router = 2 * T * H * c.num_experts
        experts = 2 * T * c.top_k * 3 * H * c.moe_intermediate_size
        head = 2 * T * H * c.vocab_size
        per_layer = qkv + o + attn + router + experts
        return {"per_layer": per_layer, "layers": c.num_layers * per_layer, "lm_head": head,
                "total": c.num_layers * per_layer + head, "experts_per_layer": experts, "attention_per_layer": attn}

    def step_flops(self, training: bool = True) -> int:
        f = self.forward_flops()["total"]
        return 3 * f if training else f

    def tflops(self, step_ms: float, training: bool = True) -> float:
        return self.step_flops(training) / (step_ms * 1e-3) / 1e12


class FlopsProfile:
    """Timed region with an analytic FLOP breakdown (the reference wraps DeepSpeed's
    FlopsProfiler the same way, src/utils_profile.py:38-50).

    ``prof = start_flops_profile(engine)``; run the forward (or training steps);
    ``end_flops_profile(prof, outdir)`` writes ``flops_profile_{rank}.txt`` with the
    per-component FLOPs, the device time and the achieved TFLOP/s of this rank.
    """

    def __init__(self, model, tokens_per_rank=None, seq_len=None, training=False, steps=1):
        self.model = getattr(model, "module", model)
        cfg = self.model.cfg
        self.tokens = tokens_per_rank or 4096
        self.counter = FlopCounter(cfg, self.tokens, seq_len or self.tokens)
        self.training, self.steps = training, steps
        self.ms = None
        if torch.cuda.is_available():
            self._s, self._e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self._s.record()
        else:
            import time

            self._t0 = time.perf_counter()

    def stop(self) -> float:
        if self.ms is None:
            if torch.cuda.is_available():
                self._e.record()
                self._e.synchronize()
                self.ms = self._s.elapsed_time(self._e)
            else:
                import time

                self.ms = (time.perf_counter() - self._t0) * 1000.0
        return self.ms

    def report(self) -> str:
        f = self.counter.forward_flops()
        mult = 3 if self.training else 1
        c = self.counter.cfg
        total, expert = count_params(self.model)
        ms = self.stop() / self.steps
        lines = [f"flops profile, rank {_rank()}: {'training step' if self.training else 'forward'}, "
                 f"{self.tokens} tokens, {c.num_layers} layers",
                 f"local params: {total / 1e9:.3f} B ({expert / 1e9:.3f} B in experts)",
                 f"{'component':<22}{'GFLOP':>14}{'share':>9}"]
        parts = {"attention (QK^T, PV)": f["attention_per_layer"] * c.num_layers,
                 "experts (SwiGLU)": f["experts_per_layer"] * c.num_layers,
                 "qkv + o projections": (f["per_layer"] - f["attention_per_layer"] - f["experts_per_layer"]
                                         - 2 * self.tokens * c.hidden_size * c.num_experts) * c.num_layers,
                 "router": 2 * self.tokens * c.hidden_size * c.num_experts * c.num_layers,
                 "lm head": f["lm_head"]}
        tot = f["total"]
        for k, v in parts.items():
            lines.append(f"{k:<22}{mult * v / 1e9:>14.1f}{v / tot:>9.1%}")
        lines.append(f"{'total':<22}{mult * tot / 1e9:>14.1f}")
        lines.append(f"device time per {'step' if self.training else 'forward'}: {ms:.3f} ms; "
                     f"achieved {mult * tot / (ms * 1e-3) / 1e12:.1f} TFLOP/s")
        return "\n".join(lines) + "\n"


def start_flops_profile(engine, tokens_per_rank=None, seq_len=None, training=False, steps=1) -> FlopsProfile:
    """Start a FLOP-profiled region on the current stream (``engine`` or a model)."""
    return FlopsProfile(engine, tokens_per_rank, seq_len, training, steps)


def end_flops_profile(prof: FlopsProfile, outdir) -> Path:
    """Stop the region and write ``flops_profile_{rank}.txt`` under ``outdir``."""
    outdir = Path(outdir)
    outdir.mkdir(parents=True, exist_ok=True)
    path = outdir / f"flops_profile_{_rank()}.txt"
    path.write_text(prof.report())
    return path


class CommLogger:
    """Per-operation count / bytes / device time of collectives and P2P transfers.

    ``with logger.op("dispatch", nbytes):`` records CUDA events around a region;
    ``summary()`` reduces latency with MAX over ranks and reports algorithm bandwidth
    (replaces DeepSpeed's comms logger, scripts/ds_moe.py:136-143).
    """

    def __init__(self):
        self.events: dict[str, list] = {}

    class _Op:
        def __init__(self, log, name, nbytes):
            self.log, self.name, self.nbytes = log, name, nbytes

        def __enter__(self):
            self.s = torch.cuda.Event(enable_timing=True)
            self.e = torch.cuda.Event(enable_timing=True)
            self.s.record()
            return self

        def __exit__(self, *exc):
            self.e.record()
            self.log.events.setdefault(self.name, []).append((self.s, self.e, self.nbytes))

    def op(self, name: str, nbytes: int = 0):
        return CommLogger._Op(self, name, nbytes)

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for name, evs in sorted(self.events.items()):
            ms = torch.tensor([s.elapsed_time(e) for s, e, _ in evs], dtype=torch.float64,
                              device=torch.cuda.current_device())
            if dist.is_available() and dist.is_initialized():
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            nbytes = sum(b for _, _, b in evs)
            total_ms = float(ms.sum())
            out[name] = {"count": len(evs), "bytes": nbytes, "total_ms": total_ms,
                         "avg_us": 1000 * total_ms / max(len(evs), 1),
                         "algbw_GBps": nbytes / (total_ms * 1e-3) / 1e9 if total_ms > 0 else 0.0}
        return out


_STAGE_RANGES = os.environ.get("SEPX_NVTX", "0") == "1"


def enable_stage_ranges(on: bool = True):
    """Turn the NVTX / profiler ranges of :func:`stage` on or off."""
    global _STAGE_RANGES
    _STAGE_RANGES = bool(on)


@contextlib.contextmanager
def stage(name: str):
    """NVTX range + torch.profiler label around one stage, and device timestamps when a
    :class:`spec_ep.utils.trace.DeviceTimeline` is enabled (no-op otherwise)."""
    from .trace import active_timeline

    tl = active_timeline()
    if not _STAGE_RANGES and tl is None:
        yield
        return
    if tl is not None:
        tl.mark(name + ":begin")
    if _STAGE_RANGES:
        torch.cuda.nvtx.range_push(name)
    try:
        if _STAGE_RANGES:
            with record_function(name):
                yield
        else:
            yield
    finally:
        if _STAGE_RANGES:
            torch.cuda.nvtx.range_pop()
        if tl is not None:
            tl.mark(name + ":end")
