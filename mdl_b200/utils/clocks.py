"""GPU clock / throttle sampling during a timed region (``nvidia-smi -lms``)."""

from __future__ import annotations

import os
import shutil
import signal
import statistics
import subprocess
import tempfile

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """Starts ``nvidia-smi`` sampling every ``period_ms`` on one GPU; ``stop()`` returns a summary."""

    def __init__(self, gpu_index: int, period_ms: int = 200) -> None:
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="mdl_clocks_", suffix=".csv")
        os.close(fd)
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen([exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                                      f"-lms={self.period_ms}", f"--id={self.gpu_index}"],
                                     stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.send_signal(signal.SIGTERM)
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._fh.close()
        sm, smax, power, reasons = [], [], [], set()
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for name, flag in zip(REASONS, parts[5:9]):
                    if flag.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "power_w_max": max(power),
                "samples": len(sm), "reasons": sorted(reasons)}
