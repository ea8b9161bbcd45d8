"""GPU clock / throttle sampling during a timed region.

Samples SM clock, max SM clock, power and the clock-event (throttle) reasons of one
GPU from a background thread through NVML (read-only queries; nothing is set), every
``period_ms`` and once right at start and stop, so even a timed region of a few tens
of milliseconds gets samples. Falls back to ``nvidia-smi -lms`` when NVML is not
importable.
"""

from __future__ import annotations

import os
import shutil
import signal
import statistics
import subprocess
import tempfile
import threading

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
# NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
_NVML_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}


def _summary(sm, smax, power, reasons) -> dict:
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "power_w_max": max(power) if power else None,
            "samples": len(sm), "reasons": sorted(reasons)}


class _NvmlSampler:
    def __init__(self, gpu, period_ms: int) -> None:
        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        if isinstance(gpu, str) and gpu.startswith("GPU-"):
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(gpu)
        else:
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(int(gpu))
        self.period = period_ms / 1000.0
        self.sm, self.smax, self.power, self.reasons = [], [], [], set()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _sample(self) -> None:
        nv, h = self.nv, self.handle
        try:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            try:
                power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            except nv.NVMLError:
                power = None
            get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            bits = int(get(h))
        except nv.NVMLError:
            return
        self.sm.append(float(sm))
        self.smax.append(float(smax))
        if power is not None:
            self.power.append(power)
        for name, bit in _NVML_BITS.items():
            if bits & bit:
                self.reasons.add(name)

    def _run(self) -> None:
        while not self._stop.wait(self.period):
            self._sample()

    def start(self) -> None:
        self._sample()
        self._thread.start()

    def stop(self) -> dict:
        self._sample()
        self._stop.set()
        self._thread.join(timeout=5)
        out = _summary(self.sm, self.smax, self.power, self.reasons)
        try:
            self.nv.nvmlShutdown()
        except Exception:  # noqa: BLE001 - shutdown failures do not matter here
            pass
        out["source"] = "nvml"
        return out


class ClockSampler:
    """Samples one GPU (index or ``GPU-<uuid>``) during a timed region; ``stop()`` returns a summary."""

    def __init__(self, gpu_index, period_ms: int = 10) -> None:
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None
        self._nvml = None

    def start(self) -> "ClockSampler":
        try:
            self._nvml = _NvmlSampler(self.gpu_index, self.period_ms)
            self._nvml.start()
            return self
        except Exception:  # noqa: BLE001 - NVML missing or no such GPU: use nvidia-smi
            self._nvml = None
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="mdl_clocks_", suffix=".csv")
        os.close(fd)
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen([exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                                      f"-lms={max(self.period_ms, 50)}", f"--id={self.gpu_index}"],
                                     stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict:
        if self._nvml is not None:
            return self._nvml.stop()
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
        out = _summary(sm, smax, power, reasons)
        out["source"] = "nvidia-smi"
        return out
