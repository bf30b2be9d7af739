"""Device-side stage timeline (per-rank ring buffer of device timestamps).

``DeviceTimeline.mark(name)`` launches a one-thread kernel that appends
``(tag, %globaltimer ns)`` to a ring buffer on the current stream, so a stage's begin and
end are stamped where the GPU actually runs them (the kernels of a stage may still be
queued when the host leaves it). ``with timeline.span(name):`` stamps both ends;
``enable_stage_timeline(timeline)`` makes every :func:`spec_ep.utils.profile.stage` of the
EP layer (dispatch, experts, combine, their backward halves, the expert weight
gradients) do so. ``durations()`` pairs the stamps into per-stage totals; with
``max_over_ranks=True`` each stage's total is the maximum over the ranks of the default
process group (every rank must call it). Timestamps from different GPUs are not
compared with each other: only differences taken on one GPU are reported.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class DeviceTimeline:
    def __init__(self, capacity: int = 8192, device=None):
        from ..ops._ext import load

        self._C = load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.capacity = int(capacity)
        self.ring = torch.zeros(self.capacity, 2, dtype=torch.int64, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.names: list[str] = []
        self._tag: dict[str, int] = {}

    def _tag_of(self, name: str) -> int:
        t = self._tag.get(name)
        if t is None:
            t = self._tag[name] = len(self.names)
            self.names.append(name)
        return t

    def mark(self, name: str):
        """Stamp ``name`` on the current stream (2 * tag = begin, 2 * tag + 1 = end)."""
        self._C.trace_stamp(self.ring, self.counter, self._tag_of(name))

    def span(self, name: str):
        tl = self

        class _Span:
            def __enter__(self):
                tl.mark(name + ":begin")

            def __exit__(self, *exc):
                tl.mark(name + ":end")

        return _Span()

    def reset(self):
        self.counter.zero_()
        self.ring.zero_()

    def events(self) -> list[tuple[str, int]]:
        """(name, device ns) in stamp order (synchronises the device)."""
        torch.cuda.synchronize(self.device)
        n = int(self.counter.item())
        ring = self.ring.cpu()
        if n > self.capacity:  # wrapped: the oldest entries were overwritten
            order = list(range(n % self.capacity, self.capacity)) + list(range(n % self.capacity))
        else:
            order = list(range(n))
        return [(self.names[int(ring[i, 0])], int(ring[i, 1])) for i in order]

    def durations(self, max_over_ranks: bool = False) -> dict:
        """Per stage: number of spans and total / mean device µs (begin..end pairs)."""
        open_at: dict[str, list[int]] = {}
        acc: dict[str, list[float]] = {}
        for name, t in self.events():
            base, _, edge = name.rpartition(":")
            if edge == "begin":
                open_at.setdefault(base, []).append(t)
            elif edge == "end" and open_at.get(base):
                acc.setdefault(base, []).append((t - open_at[base].pop()) / 1000.0)
        stages = sorted(acc)
        if max_over_ranks and dist.is_available() and dist.is_initialized():
            allnames = [None] * dist.get_world_size()
            dist.all_gather_object(allnames, stages)
            stages = sorted({s for lst in allnames for s in lst})
            tot = torch.tensor([sum(acc.get(s, [])) for s in stages], dtype=torch.float64, device=self.device)
            dist.all_reduce(tot, op=dist.ReduceOp.MAX)
            totals = tot.tolist()
        else:
            totals = [sum(acc[s]) for s in stages]
        out = {}
        for s, total in zip(stages, totals):
            n = len(acc.get(s, []))
            out[s] = {"count": n, "total_us": total, "mean_us": total / max(n, 1)}
        return out


_ACTIVE: DeviceTimeline | None = None


def enable_stage_timeline(timeline: DeviceTimeline | None):
    """Route every ``stage(name)`` through ``timeline.span(name)`` (None turns it off)."""
    global _ACTIVE
    _ACTIVE = timeline


def active_timeline() -> DeviceTimeline | None:
    return _ACTIVE
