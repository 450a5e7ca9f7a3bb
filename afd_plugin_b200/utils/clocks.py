"""Sample GPU clocks and throttle reasons while a timed region runs.

Reads ``nvidia-smi --query-gpu ... -lms 200`` into a temporary file and
summarises it (median SM MHz under load, max SM MHz, active throttle
reasons).  Only reads settings; never changes them.
"""

from __future__ import annotations

import csv
import os
import shutil
import statistics
import subprocess
import tempfile

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int = 0, period_ms: int = 200):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def __enter__(self) -> "ClockSampler":
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits", f"-i={self.gpu_index}",
             f"-lms={self.period_ms}"],
            stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._fh.close()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        rows = []
        with open(self.path) as fh:
            for rec in csv.reader(fh):
                if len(rec) < 9:
                    continue
                try:
                    rows.append([x.strip() for x in rec])
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(rows),
        }


__all__ = ["ClockSampler"]
