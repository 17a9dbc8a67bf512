"""SM-clock and throttle-reason sampling during a timed region (NVML, read-only).

A background thread polls NVML every few milliseconds while device work is
timed, so every measured rate can be read against the clock it ran at.  Only
queries are made; no clock, power or other device setting is changed.
"""

from __future__ import annotations

import os
import statistics
import threading
import time

# NVML clocks-event (throttle) reason bits.
REASONS = {
    0x0000000000000001: "gpu_idle",
    0x0000000000000002: "applications_clocks_setting",
    0x0000000000000004: "sw_power_cap",
    0x0000000000000008: "hw_slowdown",
    0x0000000000000020: "sw_thermal_slowdown",
    0x0000000000000040: "hw_thermal_slowdown",
    0x0000000000000080: "hw_power_brake_slowdown",
    0x0000000000000100: "display_clock_setting",
}
REJECTING = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def _physical_index(device_index: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        entries = [v for v in visible.split(",") if v.strip()]
        if device_index < len(entries) and entries[device_index].strip().isdigit():
            return int(entries[device_index])
    return device_index


class ClockSampler:
    """Context manager: samples SM clock, power and throttle reasons while open."""

    def __init__(self, device_index: int = 0, period_s: float = 0.002):
        self.period = period_s
        self.samples: list[int] = []
        self.power_mw: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(_physical_index(device_index))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # noqa: BLE001 - reported as unavailable
            self._nvml = None
            self.error = str(exc)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.reasons.update(name for bit, name in REASONS.items()
                                    if mask & bit and name != "gpu_idle")
                self.power_mw.append(nv.nvmlDeviceGetPowerUsage(self._handle))
            except Exception:  # noqa: BLE001 - a missed sample is not an error
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0, "source": "nvml", "error": self.error}
        return {"sm_mhz": statistics.median(self.samples), "sm_min_mhz": min(self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "power_w_max": max(self.power_mw) / 1000 if self.power_mw else None,
                "samples": len(self.samples), "source": "nvml",
                "rejected": any(r in self.reasons for r in REJECTING)}
