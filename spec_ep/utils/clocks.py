"""Sample SM clocks and throttle reasons with nvidia-smi while a region runs (read-only)."""
from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """Runs ``nvidia-smi --query-gpu ... -lms`` for one GPU (by UUID) in the background."""

    def __init__(self, gpu_uuid: str | None, period_ms: int = 200):
        self.uuid, self.period = gpu_uuid, period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        self.out = None
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period}"]
            if self.uuid:
                cmd.insert(1, f"--id={self.uuid}")
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:  # no nvidia-smi: the summary reports the region as unsampled
            self.proc = None
            if self.out is not None:
                self.out.close()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.close()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set()
        for _, _, flags in rows:
            for name, v in zip(REASONS, flags):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}
