"""Sample SM clocks and throttle reasons with ``nvidia-smi`` while a
measured region runs (read-only queries; no setting is changed)."""

from __future__ import annotations

import os
import statistics
import subprocess
import tempfile

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int | None = None, period_ms: int = 200):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.path = None

    def start(self) -> None:
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period}"]
        if self.gpu is not None:
            cmd.insert(1, f"--id={self.gpu}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        return summarize_clock_rows(rows)


def summarize_clock_rows(rows: list[list[str]]) -> dict:
    def num(x):
        try:
            return float(x)
        except ValueError:
            return None

    sm = [num(r[1]) for r in rows if num(r[1]) is not None]
    smax = [num(r[2]) for r in rows if num(r[2]) is not None]
    power = [num(r[3]) for r in rows if num(r[3]) is not None]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = set()
    for r in rows:
        for i, n in enumerate(names):
            if r[5 + i].lower().startswith("active"):
                reasons.add(n)
    load = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
    return {
        "sm_mhz": statistics.median(load) if load else None,
        "sm_max_mhz": max(smax) if smax else None,
        "reasons": sorted(reasons),
        "samples": len(rows),
        "power_w_max": max(power) if power else None,
    }
