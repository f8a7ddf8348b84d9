"""Background ``nvidia-smi`` sampler of SM clocks and throttle reasons, used
to qualify benchmark numbers (read-only queries; no GPU setting is changed)."""
from __future__ import annotations

import os
import signal
import statistics
import subprocess
import tempfile
from typing import Optional

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_indices: Optional[list[int]] = None, period_ms: int = 200):
        self.gpus = gpu_indices
        self.period_ms = period_ms
        self.proc: Optional[subprocess.Popen] = None
        self.path: Optional[str] = None

    def start(self) -> None:
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
        if self.gpus:
            cmd.insert(1, "-i=" + ",".join(str(g) for g in self.gpus))
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
                                         start_new_session=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is not None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)
            except (ProcessLookupError, PermissionError):
                pass
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                pass
        return self.summary()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(_REASONS, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
            os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}
