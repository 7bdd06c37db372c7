"""Sample GPU clocks and throttle reasons with nvidia-smi during a timed region.

Only reads settings; nothing here changes a GPU's clocks or limits.
"""
from __future__ import annotations

import shutil
import subprocess
import tempfile
import statistics

_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int = 0, period_ms: int = 200):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.file = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits",
             "-i", str(self.gpu_index), "-lms", str(self.period_ms)],
            stdout=self.file, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        with open(self.file.name) as fh:
            rows = [line.strip().split(", ") for line in fh if line.strip()]
        sm, sm_max, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for row in rows:
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                sm_max.append(float(row[2]))
            except ValueError:
                continue
            for name, value in zip(names, row[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(sm_max),
                "reasons": sorted(reasons), "samples": len(sm)}
